#!/usr/bin/env python3
"""Benchmark of the B200 back end on the reference's headline workload.

Metric: pixels/s (and tiles/hour) of the Tessera v2 Large
pixel-student encoder. One step = one full encode of the workload tile: device
binning, padding and standardisation, both backbones, the fusion head and the
int8 quantisation, for every pixel.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference|refcuda]

* N = 1: config 1, the Manchester-sized synthetic tile (1113 x 695 px,
  T2 = 120 at 60% valid, Ta = Td = 60), seeded; Large weights random-init from
  seed 0 (Xavier-uniform, zero biases).
* N > 1 (under torchrun, one process per GPU): config 2, the same tile split by
  pixel rows (FLOP-balanced) across the ranks; no inter-GPU traffic on the data
  path (a barrier and a max-reduce of the timings only). Total work is fixed,
  so scaling is "strong". With --config 4, each rank encodes its own whole
  tile instead (config 4's batch of tiles, one per GPU; scaling "weak").
* `value` is the whole-job throughput with the tile already resident in HBM;
  `e2e` is the same through tc_encode_tile_rows with pinned host buffers
  (host->device copy of the rank's rows and device->host copy of codes and
  scales inside every timed step).
* The tile (2.2 GB) is larger than the 126 MB L2, so no flush is needed
  between steps.
* --impl reference: the reference's own driver (src/tessera_encode.cpp,
  unmodified) with the CPU back-end restatement (oracle/_ref/tessera_encode_ref)
  on all host cores, on bounded pixel samples of the same tile; rank 0 only.
* --impl refcuda: the reference's own driver + CUDA back end (cuBLASLt)
  rebuilt for sm_100a (oracle/_ref/tessera_encode_cuda_ref) on one B200, on the
  whole tile through its CLI (load from disk included, as the reference times it).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path[:0] = [str(REPO / "tessera-inference_b200"), str(REPO / "oracle")]

import synth  # noqa: E402

METRIC = "pixels/sec (tiles/hour) per B200 and whole box at 1/2/4/8 GPUs vs ref CPU"
UNIT = "px/s"
WORKLOAD = "config 1: synthetic Manchester-sized tile 1113x695 (773,535 px), T2=120 (60% valid), Ta=Td=60"
# DRAM bytes per GEMM FLOP: dram__bytes_read.sum + dram__bytes_write.sum summed
# over the 1,587 GEMM launches of one ncu capture of a config-1 band (64 rows of
# a tile with config 1's series and value distributions; 842.0 GB for 3.751e14
# FLOP; profiles/launch_list_config1_band.md), and the algorithmic bytes per
# FLOP of the same launches (per token emb2 2,560 B and per layer QKV 5,120 B,
# out-proj 3,840 B, FFN1 6,400 B, FFN2 7,680 B; 8.851e11 B).
GEMM_DRAM_BYTES_PER_FLOP = 2.245e-3
GEMM_ALG_BYTES_PER_FLOP = 2.36e-3
SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


def measured_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons of one GPU, sampled every 200 ms."""

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None
        self.f = None

    def __enter__(self):
        self.f = tempfile.TemporaryFile(mode="w+")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={SMI_FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.gpu_id], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.f is None:
            return {}
        self.f.seek(0)
        sm, mx, reasons, n = [], 0.0, set(), 0
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                s, m, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            n += 1
            mx = max(mx, m)
            if pw > 200.0:  # under load
                sm.append(s)
            for name, v in zip(REASONS, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": n, "samples_under_load": len(sm)}


def weights_file(tmp: Path) -> Path:
    return synth.make_weights(tmp / "student_large_seed0.tcw", seed=0)


def band_arrays(tile: dict, r0: int, r1: int) -> dict:
    """Rows [r0, r1) of every per-pixel array (all time steps), contiguous."""
    out = dict(tile)
    for k in ("bands", "masks", "asc", "desc"):
        out[k] = np.ascontiguousarray(tile[k][:, r0:r1])
    return out


def rank_rows(tile: dict, rank: int, world: int) -> tuple[int, int]:
    """This rank's row band: FLOP-balanced contiguous rows (tc_plan_rows)."""
    import tessera_b200 as tb
    bounds = tb.plan_rows(tile, world)
    return bounds[rank], bounds[rank + 1]


def tile_bytes(t: dict) -> int:
    return sum(int(v.nbytes) for v in t.values())


# ------------------------------------------------------------------ CPU reference arm
# The reference driver's own timing line (src/tessera_encode.cpp:366-370).
ENCODE_RE = re.compile(r"load=([\d.]+)s bin=([\d.]+)s prep=([\d.]+)s net=([\d.]+)s quant\+write=([\d.]+)s "
                       r"total=([\d.]+)s")


def run_ref_driver(binary: Path, tile: dict, pixels: np.ndarray, weights: Path, work: Path, threads: int) -> dict:
    """Runs a reference driver binary on the given flat pixels of the tile,
    gathered into a 1 x K tile (exact: each pixel's result depends only on its
    own series). Returns the process wall time and the driver's own ENCODE
    timings: net = tc_encode calls only, total = the whole driver run (tile
    load, binning, prep, network, quantisation, .npy write)."""
    sub = synth.subset_tile(tile, pixels)
    tdir = synth.write_tile_dir(sub, work / "grid_sample")
    # TC_BLOCK / TC_BLOCK_S2 are the reference's block sizes (pixels per OpenMP
    # task, tessera_cpu.cpp:486-489); one pixel per task keeps every core busy
    # on a sample of a few thousand pixels, whose per-key batches are small.
    env = dict(os.environ, OMP_NUM_THREADS=str(threads), OMP_PROC_BIND="close", OMP_WAIT_POLICY="ACTIVE",
               TC_BLOCK="1", TC_BLOCK_S2="1", TC_BATCH="4096")
    t0 = time.perf_counter()
    r = subprocess.run([str(binary), str(tdir), str(work / "out"), str(weights)], env=env, capture_output=True,
                       text=True, check=True)
    wall = time.perf_counter() - t0
    line = next((l for l in r.stdout.splitlines() if l.startswith("ENCODE")), "")
    m = ENCODE_RE.search(line)
    if not m:
        raise RuntimeError(f"no ENCODE timing line from {binary.name}: {r.stdout[-500:]}")
    load, bin_, prep, net, quant, total = (float(x) for x in m.groups())
    return {"px": int(len(pixels)), "wall_s": wall, "net_s": net, "total_s": total, "prep_s": prep,
            "load_s": load, "quant_write_s": quant, "line": line}


def band_pixels(tile: dict, r0: int, nrows: int) -> np.ndarray:
    """Flat indices of the contiguous row band [r0, r0 + nrows)."""
    W = tile["masks"].shape[2]
    return np.arange(r0 * W, (r0 + nrows) * W, dtype=np.int64)


def cpu_band_rows(binary, tile, weights, work, threads, target_s: float) -> tuple[int, float]:
    """Rows per band so that one run's network time is about target_s: a
    64-pixel calibration run's network-only rate (its process start and weight
    load are outside `net`)."""
    T2, H, W = tile["masks"].shape
    r = run_ref_driver(binary, tile, band_pixels(tile, H // 2, 1)[:64], weights, work, threads)
    rate = 64 / max(r["net_s"], 0.05)
    rows = int(min(max(round(target_s * rate / W), 1), H))
    return rows, rate


def cpu_summary(runs: list) -> dict:
    px = sum(r["px"] for r in runs)
    net, total, wall = (sum(r[k] for r in runs) for k in ("net_s", "total_s", "wall_s"))
    return {"px": px, "net_px_s": px / net, "total_px_s": px / total, "wall_px_s": px / wall,
            "fixed_cost_frac": (wall - net) / wall}


def cpu_reference_arm(args, tile, weights, work) -> dict:
    binary = REPO / "oracle" / "_ref" / "tessera_encode_ref"
    if not binary.exists():
        return {"impl": "reference", "unavailable": f"{binary.relative_to(REPO)} not built (make -C oracle)"}
    threads = os.cpu_count() or 1
    T2, H, W = tile["masks"].shape
    rows, _ = cpu_band_rows(binary, tile, weights, work, threads, target_s=args.cpu_step_s)
    # each step: the next contiguous band of rows, from the middle of the tile
    starts = [(H // 3 + i * rows) % max(H - rows + 1, 1) for i in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        run_ref_driver(binary, tile, band_pixels(tile, starts[i], rows), weights, work, threads)
    runs = [run_ref_driver(binary, tile, band_pixels(tile, starts[args.warmup + i], rows), weights, work, threads)
            for i in range(args.steps)]
    sm = cpu_summary(runs)
    value = sm["total_px_s"]
    sample = (f"{args.steps} steps, each a contiguous band of {rows} rows ({rows * W} px) of the config-1 tile run "
              f"as a 1x{rows * W} tile through the reference driver src/tessera_encode.cpp (unmodified) with the "
              f"C++ restatement of the oneDNN CPU back end (oneDNN is not installed), TC_BLOCK=TC_BLOCK_S2=1; "
              f"value = px / the driver's own total= time (load, bin, prep, network, quant, write); "
              f"network-only {sm['net_px_s']:.1f} px/s; fixed cost {100 * sm['fixed_cost_frac']:.1f}% of wall")
    cpu = {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample,
           "cpu_model": cpu_model(), **sm}
    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * statistics.mean(r["total_s"] for r in runs),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": {"workload": WORKLOAD, "sample_px_per_step": rows * W,
                                             "sample_rows_per_step": rows},
            "impl": "reference", "cpu_baseline": cpu, "tiles_per_hour": 3600 * value / (H * W),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_baseline_leg(tile, weights, work, target_s: float) -> dict | None:
    """The reported CPU baseline of the B200 arm: one contiguous band of rows
    (about target_s of network time on all host cores), network-only and
    whole-driver rates from the driver's own timing line."""
    binary = REPO / "oracle" / "_ref" / "tessera_encode_ref"
    if not binary.exists():
        return None
    threads = os.cpu_count() or 1
    T2, H, W = tile["masks"].shape
    rows, _ = cpu_band_rows(binary, tile, weights, work, threads, target_s=target_s)
    r = run_ref_driver(binary, tile, band_pixels(tile, H // 2, rows), weights, work, threads)
    sm = cpu_summary([r])
    return {"value": sm["total_px_s"], "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"rows {H // 2}..{H // 2 + rows - 1} ({rows * W} px, contiguous) of the config-1 tile as a "
                      f"1x{rows * W} tile through the reference driver (unmodified) + C++ restatement of the oneDNN "
                      f"CPU back end, TC_BLOCK=TC_BLOCK_S2=1; value = px / total= ({r['total_s']:.1f} s), "
                      f"network-only {sm['net_px_s']:.1f} px/s ({r['net_s']:.1f} s)",
            "cpu_model": cpu_model(), **sm}


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ------------------------------------------------------------------ reference CUDA arm
def refcuda_arm(args, tile, weights, work) -> dict:
    binary = REPO / "oracle" / "_ref" / "tessera_encode_cuda_ref"
    if not binary.exists():
        return {"impl": "refcuda", "unavailable": f"{binary.relative_to(REPO)} not built (make -C oracle cuda-ref)"}
    tdir = synth.write_tile_dir(tile, work / "grid_cfg1")
    best = None
    for chunk in (64, 512, 1024):
        env = dict(os.environ, TC_CHUNK=str(chunk), OMP_NUM_THREADS=str(os.cpu_count() or 1))
        nets, totals = [], []
        for i in range(args.warmup + args.steps):
            r = subprocess.run([str(binary), str(tdir), str(work / "out"), str(weights)], env=env,
                               capture_output=True, text=True, check=True)
            line = next(l for l in r.stdout.splitlines() if l.startswith("ENCODE"))
            if i >= args.warmup:
                nets.append(float(re.search(r"net=([\d.]+)s", line).group(1)))
                totals.append(float(re.search(r"total=([\d.]+)s", line).group(1)))
        res = {"chunk": chunk, "net_s": statistics.median(nets), "total_s": statistics.median(totals)}
        if best is None or res["total_s"] < best["total_s"]:
            best = res
    N = tile["masks"].shape[1] * tile["masks"].shape[2]
    return {"metric": METRIC, "value": N / best["total_s"], "unit": UNIT, "n_gpus": 1, "impl": "refcuda",
            "config": {"workload": WORKLOAD, "TC_CHUNK": best["chunk"]}, "net_px_s": N / best["net_s"],
            "ms_per_step": 1000 * best["total_s"], "higher_is_better": True}


def gpu_reference_leg(tile, weights, work, chunk: int = 1024, runs: int = 3) -> dict | None:
    """The reference's own CUDA back end (src/tessera_cuda.cu, cuBLASLt, rebuilt
    for sm_100a) behind its own driver on the same tile and weights: one
    warm-up run and `runs` timed runs at TC_CHUNK=chunk (its fastest setting
    on this tile), about a minute in all. net = its tc_encode calls (H2D,
    network, D2H), total = the whole driver run including the tile load."""
    binary = REPO / "oracle" / "_ref" / "tessera_encode_cuda_ref"
    if not binary.exists():
        return None
    tdir = synth.write_tile_dir(tile, work / "grid_cfg1")
    env = dict(os.environ, TC_CHUNK=str(chunk), OMP_NUM_THREADS=str(os.cpu_count() or 1))
    nets, totals = [], []
    for i in range(1 + runs):
        r = subprocess.run([str(binary), str(tdir), str(work / "out_refcuda"), str(weights)], env=env,
                           capture_output=True, text=True, check=True, timeout=120)
        m = ENCODE_RE.search(next(l for l in r.stdout.splitlines() if l.startswith("ENCODE")))
        if i > 0:
            nets.append(float(m.group(4)))
            totals.append(float(m.group(6)))
    N = tile["masks"].shape[1] * tile["masks"].shape[2]
    return {"net_px_s": N / statistics.median(nets), "total_px_s": N / statistics.median(totals), "chunk": chunk,
            "runs": runs, "net_s": nets, "total_s": totals,
            "what": "reference driver + src/tessera_cuda.cu (cuBLASLt) rebuilt for sm_100a, same tile and weights; "
                    "median of the timed runs after one warm-up"}


# ------------------------------------------------------------------ B200 arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "refcuda"])
    ap.add_argument("--config", type=int, default=1, choices=[0, 1, 3, 4])
    ap.add_argument("--cpu-step-s", type=float, default=6.0, help="network seconds per CPU reference step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpu-reference", action="store_true", help="skip the reference CUDA back-end leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg (sweeps only)")
    ap.add_argument("--profile", action="store_true", help="print the per-category TCPROF table")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        ap.error("--warmup must be >= 3")

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    work = Path(tempfile.mkdtemp(prefix="tcb_bench_"))
    weights = weights_file(work)

    if args.impl in ("reference", "refcuda"):
        if rank != 0:
            return
        tile = synth.make_config_tile(args.config)
        out = cpu_reference_arm(args, tile, weights, work) if args.impl == "reference" else refcuda_arm(
            args, tile, weights, work)
        print(json.dumps(out), flush=True)
        return

    import torch
    import tessera_b200 as tb

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))

    # config 4 is a batch of tiles, one whole tile per GPU (seed 4 + rank): the
    # work per GPU is fixed as N grows; the other configs split one tile by rows
    replicas = args.config == 4 and world > 1
    tile = synth.make_config_tile(args.config, seed=4 + rank) if replicas else synth.make_config_tile(args.config)
    T2, H, W = tile["masks"].shape
    Ta, Td = tile["asc"].shape[0], tile["desc"].shape[0]
    r0, r1 = (0, H) if replicas else rank_rows(tile, rank, world)
    band = band_arrays(tile, r0, r1)
    R = r1 - r0
    npx_band = R * W

    enc = tb.Encoder(weights)
    stream = torch.cuda.current_stream()
    enc.set_stream(stream.cuda_stream)
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in band.items()}
    codes_d = torch.empty((R, W, 128), dtype=torch.int8, device="cuda")
    scales_d = torch.empty((R, W), dtype=torch.float32, device="cuda")

    def step_device():
        enc.encode_tile_device(dev, T2, Ta, Td, R, W, 0, R, codes_d, scales_d)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step_device()
    gpu_uuid = str(torch.cuda.get_device_properties(local).uuid)
    gpu_id = gpu_uuid if gpu_uuid.startswith("GPU-") else f"GPU-{gpu_uuid}"
    enc.reset_stats()
    barrier()
    with ClockSampler(gpu_id) as clocks:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step_device()
        e1.record(stream)
        torch.cuda.synchronize()
        dev_ms = e0.elapsed_time(e1)
    barrier()
    launches = enc.stats()["launches"]
    dev_ms_max = max_over_ranks(dev_ms)

    # one more step with per-launch CUDA events (category timing, GEMM roofline)
    enc.reset_stats()
    enc.set_profiling(True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    step_device()
    e1.record(stream)
    torch.cuda.synchronize()
    prof_ms = e0.elapsed_time(e1)
    st = enc.stats()
    enc.set_profiling(False)
    if args.profile:
        enc.profile_dump()
    barrier()

    # end to end: host (pinned) -> device -> host, through tc_encode_tile_rows
    e2e_ms_max, e2e_ms, ok = None, None, None
    if not args.no_e2e:
        pin = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in band.items()}
        pin_np = {k: v.numpy() for k, v in pin.items()}
        codes_h = torch.empty((R, W, 128), dtype=torch.int8).pin_memory().numpy()
        scales_h = torch.empty((R, W), dtype=torch.float32).pin_memory().numpy()
        for _ in range(args.warmup):
            enc.encode_tile(pin_np, 0, R, codes_h, scales_h)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            enc.encode_tile(pin_np, 0, R, codes_h, scales_h)
        e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1)
        e2e_ms_max = max_over_ranks(e2e_ms)
        barrier()
        # the device-resident and host-buffer paths must give the same bytes
        ok = bool(np.array_equal(codes_d.cpu().numpy(), codes_h)) and bool(
            np.array_equal(scales_d.cpu().numpy().view(np.uint32), scales_h.view(np.uint32)))

    # per-rank device times and row bands (under torchrun every rank takes part)
    mine = [dev_ms, e2e_ms if e2e_ms is not None else -1.0, float(r0), float(r1)]
    if dist is not None:
        t = torch.tensor(mine, dtype=torch.float64, device="cuda")
        allv = torch.zeros(world * len(mine), dtype=torch.float64, device="cuda")
        dist.all_gather_into_tensor(allv, t)
        per_rank = allv.view(world, len(mine)).cpu().tolist()
    else:
        per_rank = [mine]

    tile_px = H * W
    total_px = tile_px * (world if replicas else 1)  # pixels the whole job processes per step
    value = total_px * args.steps / (dev_ms_max / 1000.0)
    e2e_value = total_px * args.steps / (e2e_ms_max / 1000.0) if e2e_ms_max else None
    h2d = tile_bytes(band)
    d2h = npx_band * 128 + npx_band * 4

    peaks = measured_peaks()
    cat = st["ms_cat"]
    gemm_ms = cat["gemm"]
    gemm_tflops = st["gemm_flop"] / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
    peak = peaks["bf16_sustained"]
    alg_tflops = st["alg_flop"] * args.steps / (dev_ms * 1e-3) / 1e12

    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_leg(tile, weights, work, target_s=20.0)
    gpu_ref = None
    if world == 1 and args.config == 1 and not args.no_gpu_reference:
        gpu_ref = gpu_reference_leg(tile, weights, work)
    out = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak" if replicas else "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD if args.config == 1 else f"config {args.config}",
                   "chunk_tokens": int(os.environ.get("TC_CHUNK_TOKENS", "524288")),
                   "pixels": total_px,
                   "split": (f"one whole tile per GPU (seeds 4..{3 + world})" if replicas
                             else f"rows FLOP-balanced over {world} GPU(s)"),
                   "weights": "Large, Xavier-uniform seed 0, zero biases",
                   "l2": f"inputs ({tile_bytes(band) / 1e9:.1f} GB per GPU) larger than L2; no flush"},
        "tiles_per_hour": 3600.0 * value / tile_px,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                "tiles_per_hour": 3600.0 * e2e_value / tile_px if e2e_value else None},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "kernel": "k_gemm_bf16 / k_gemm_bf16_tn (tcgen05)",
                     "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s",
                     "frac": gemm_tflops / peak if gemm_tflops else None,
                     "peak_source": f"{peaks['source']} bf16 sustained (kernel timed inside a long step)",
                     "measured": "per-launch CUDA events on the library stream over one profiled step after the timed steps",
                     "traffic": (GEMM_DRAM_BYTES_PER_FLOP * st["gemm_flop"] / st["gemm_launches"]
                                 if st.get("gemm_launches") else None),
                     "traffic_unit": "DRAM bytes per GEMM launch",
                     "traffic_source": "ncu DRAM bytes per FLOP of every GEMM launch of a config-1 band "
                                       "(profiles/launch_list_config1_band.md), scaled by this run's FLOP per "
                                       "launch",
                     "algorithmic_bytes_per_launch": (GEMM_ALG_BYTES_PER_FLOP * st["gemm_flop"] / st["gemm_launches"]
                                                      if st.get("gemm_launches") else None),
                     "end_to_end_tflops": alg_tflops, "end_to_end_frac": alg_tflops / peak},
        "phase_ms_per_step": cat, "profiled_step_ms": prof_ms,
        "gemm_tflops_by_layer": {k: (v["flop"] / (v["ms"] * 1e-3) / 1e12 if v["ms"] > 0 else None)
                                 for k, v in st["gemm_kind"].items()},
        "clocks": clocks.summary(),
        "outputs_match_e2e": ok,
        "per_rank_ms": [r[0] / args.steps for r in per_rank],
        "per_rank_e2e_ms": [r[1] / args.steps if r[1] >= 0 else None for r in per_rank],
        "band_rows": [[int(r[2]), int(r[3])] for r in per_rank],
    }
    if cpu:
        out["cpu_baseline"] = cpu
    if gpu_ref:
        out["gpu_reference"] = gpu_ref
    print(json.dumps(out), flush=True)
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
