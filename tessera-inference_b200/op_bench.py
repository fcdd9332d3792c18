"""Time one back-end kernel alone on a synthetic chunk, through the library's
operator entry points (include/tessera_b200_ops.h), with CUDA events.

  python tessera-inference_b200/op_bench.py attention --T 120        # uniform series of 120 steps
  python tessera-inference_b200/op_bench.py layernorm --M 131072
  python tessera-inference_b200/op_bench.py gemm --M 524288 --N 2560 --K 640 --mode relu --seconds 3 [--torch]
  python tessera-inference_b200/op_bench.py encode --rows 64 --reps 2      # a profiling driver

Prints one JSON line: microseconds per launch, the algorithmic bytes of the
launch and the bandwidth they give. Attention bytes per token are the Q, K and
V rows read (3 x 640 bf16) and the output row written (640 bf16): 5,120 B.
LayerNorm bytes per row are 640 bf16 read and written: 2,560 B. Inputs are
seeded random bf16 in device memory, larger than L2 at the default sizes.
`TC_ATTN_TC=2` selects the tcgen05 attention kernel for every series of up
to 128 steps and `TC_ATTN_TC=0` the mma.sync kernel; unset, the library
takes tcgen05 for series longer than 48 steps and up to 128.

The chunk is described by its series length alone (no offsets array), so the
entry point does no host work and the launches run back to back.

`gemm` times the tcgen05 GEMM on one layer shape (mode: bias, relu = bias +
ReLU, res = bias + residual) for about --seconds of back-to-back launches, so
the clock settles under the power cap, and reports TFLOP/s with the median
SM clock sampled by nvidia-smi over the timed loop (and TFLOP/s per GHz).
--torch times torch.matmul (cuBLAS, bf16, no epilogue) on the same shape the
same way, as a comparison point; it is not part of the back end.

`encode` runs the whole device path (tc_encode_tile_device) --reps times on
a seeded tile of --rows rows with config 1's width, series lengths and value
distributions (synth.make_tile), so every kernel of the path launches at
config-1 chunk sizes; it is the small workload the ncu captures run.
"""
from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
import tessera_b200 as tb  # noqa: E402


def time_launches(fn, reps: int) -> float:
    """Microseconds per launch over `reps` launches after three warm-up ones."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / reps


class SmClocks:
    """Median SM clock (MHz) of the current GPU while the block runs (nvidia-smi, 100 ms samples)."""

    def __enter__(self):
        self.f = tempfile.TemporaryFile(mode="w+")
        uuid = str(torch.cuda.get_device_properties(torch.cuda.current_device()).uuid)
        gpu = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        try:
            self.p = subprocess.Popen(["nvidia-smi", "--query-gpu=clocks.sm,power.draw", "--format=csv,noheader,nounits",
                                       "-lms", "100", "-i", gpu], stdout=self.f, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.p = None
        time.sleep(0.2)
        return self

    def __exit__(self, *exc):
        if self.p is not None:
            self.p.terminate()
            self.p.wait(5)

    def median(self):
        self.f.seek(0)
        v = []
        for line in self.f.read().splitlines():
            try:
                mhz, w = (float(x) for x in line.split(","))
            except ValueError:
                continue
            if w > 300:
                v.append(mhz)
        return statistics.median(v) if v else None


def time_for(fn, seconds: float) -> tuple[float, int, float | None]:
    """(microseconds per launch, launches, median SM MHz) over about `seconds`."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    fn()
    torch.cuda.synchronize()
    reps = max(3, int(seconds / max(time.perf_counter() - t0, 1e-6)))
    with SmClocks() as clk:
        us = time_launches(fn, reps)
    return us, reps, clk.median()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("op", choices=["attention", "layernorm", "gemm", "encode"])
    ap.add_argument("--rows", type=int, default=64, help="tile rows (encode)")
    ap.add_argument("--N", type=int, default=2560)
    ap.add_argument("--K", type=int, default=640)
    ap.add_argument("--mode", choices=["bias", "relu", "res"], default="relu")
    ap.add_argument("--variant", type=int, default=0, help="0 per-layer choice, 1 single CTA, 2 CTA pair, 3 operand-swapped")
    ap.add_argument("--seconds", type=float, default=3.0)
    ap.add_argument("--torch", action="store_true", help="also time torch.matmul (cuBLAS) on the same shape")
    ap.add_argument("--T", type=int, default=120, help="uniform series length (attention)")
    ap.add_argument("--tokens", type=int, default=131072, help="tokens per attention chunk")
    ap.add_argument("--M", type=int, default=131072, help="rows (layernorm)")
    ap.add_argument("--reps", type=int, default=10)
    a = ap.parse_args(argv)
    lib = tb.load_library()
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(0)
    if a.op == "attention":
        npix = a.tokens // a.T
        M = npix * a.T
        qkv = torch.randn(M, 1920, device="cuda", generator=g).to(torch.bfloat16)
        att = torch.empty(M, 640, device="cuda", dtype=torch.bfloat16)

        def run():
            if lib.tcb_op_attention(qkv.data_ptr(), None, a.T, npix, a.T, att.data_ptr(), st):
                raise RuntimeError("tcb_op_attention failed")

        us = time_launches(run, a.reps)
        nbytes = M * 5120
        rec = {"op": "attention", "tokens": M, "pixels": npix, "T": a.T}
    elif a.op == "encode":
        import tempfile as tf
        import synth
        tile = synth.make_tile(H=a.rows, W=695, T2=120, Ta=60, Td=60, p=0.6, seed=2)
        T2, H, W = tile["masks"].shape
        with tf.TemporaryDirectory() as td:
            enc = tb.Encoder(synth.make_weights(Path(td) / "w.tcw", seed=0))
        dev = {k: torch.from_numpy(v).cuda() for k, v in tile.items()}
        codes = torch.empty((H, W, 128), dtype=torch.int8, device="cuda")
        scales = torch.empty((H, W), dtype=torch.float32, device="cuda")
        enc.set_stream(st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(a.reps):
            if i == a.reps - 1:
                e0.record()
            enc.encode_tile_device(dev, T2, 60, 60, H, W, 0, H, codes, scales)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        enc.close()
        print(json.dumps({"op": "encode", "pixels": H * W, "ms_last": round(ms, 2), "px_s": round(H * W / ms * 1e3)}))
        return 0
    elif a.op == "gemm":
        M, N, K = a.M, a.N, a.K
        A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        W = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
        bias = torch.randn(N, device="cuda", generator=g) * 0.1
        res = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16) if a.mode == "res" else None
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")

        def run():
            if lib.tcb_op_gemm(A.data_ptr(), K, W.data_ptr(), bias.data_ptr(), int(a.mode == "relu"),
                               res.data_ptr() if res is not None else None, N, None, 1, None, None, out.data_ptr(), N,
                               M, N, K, 0, a.variant, status.data_ptr(), st):
                raise RuntimeError("tcb_op_gemm failed")

        us, reps, mhz = time_for(run, a.seconds)
        torch.cuda.synchronize()
        if status.item() != 0:
            raise RuntimeError(f"device status {status.item()}")
        flop = 2.0 * M * N * K
        rec = {"op": "gemm", "M": M, "N": N, "K": K, "mode": a.mode, "variant": a.variant,
               "us_per_launch": round(us, 2), "TFLOP_s": round(flop / us / 1e6, 1), "sm_mhz": mhz,
               "TFLOP_s_per_GHz": round(flop / us / 1e6 / (mhz / 1e3), 1) if mhz else None, "reps": reps}
        if a.torch:
            Wt = W.t()

            def run_t():
                torch.matmul(A, Wt, out=out)

            us_t, reps_t, mhz_t = time_for(run_t, a.seconds)
            rec["cublas"] = {"us_per_launch": round(us_t, 2), "TFLOP_s": round(flop / us_t / 1e6, 1), "sm_mhz": mhz_t,
                             "TFLOP_s_per_GHz": round(flop / us_t / 1e6 / (mhz_t / 1e3), 1) if mhz_t else None,
                             "reps": reps_t, "what": "torch.matmul bf16, no epilogue"}
        print(json.dumps(rec))
        return 0
    else:
        M = a.M
        x = torch.randn(M, 640, device="cuda", generator=g).to(torch.bfloat16)
        y = torch.empty_like(x)
        gam = torch.ones(640, device="cuda")
        bet = torch.zeros(640, device="cuda")

        def run():
            if lib.tcb_op_layernorm640(x.data_ptr(), M, gam.data_ptr(), bet.data_ptr(), y.data_ptr(), st):
                raise RuntimeError("tcb_op_layernorm640 failed")

        us = time_launches(run, a.reps)
        nbytes = M * 2560
        rec = {"op": "layernorm640", "rows": M}
    rec.update({"us_per_launch": round(us, 2), "bytes_per_launch": nbytes, "GB_per_s": round(nbytes / us / 1e3, 1),
                "reps": a.reps})
    print(json.dumps(rec))
    return 0


if __name__ == "__main__":
    sys.exit(main())
