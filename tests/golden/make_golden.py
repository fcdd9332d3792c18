"""Generate the golden fixtures of tests/golden/.

  python tests/golden/make_golden.py padpattern
      pad_pattern.npz: _pad_pattern(n, B) from numpy's own linspace /
      array_split (the functions src/tessera_encode.cpp:157,169 mirror).
  python tests/golden/make_golden.py driver
      For each case tile: run the reference's unmodified driver
      (oracle/_ref/tessera_encode_ref = src/tessera_encode.cpp + the CPU
      back-end restatement) with TC_ORACLE_DUMP set. Stores <case>_batches.json
      (per tc_encode call: G, T2, T1 and sha256 of the s2 / s1 records the
      reference driver prepared) and <case>_oracle.npz (the codes and scales
      it wrote).
  python tests/golden/make_golden.py export
      export_ref.json: for synth.fake_checkpoint in f32 and in bf16, the
      sha256 and size of the .tcw that the reference's unmodified
      tools/export_weights.py writes (run here, from the reference tree).
  python tests/golden/make_golden.py api
      ref_api.json: the tokens of the four back-end prototypes
      (tc_create / tc_encode / tc_profile_dump / tc_destroy) as the reference
      driver declares them (src/tessera_encode.cpp:47-52).
  python tests/golden/make_golden.py subsets [CFG ...]
      cfg1_subset.npz, cfg3_subset.npz, cfg4_subset.npz: a stratified pixel
      subset of the full-size benchmark tiles of configs 1, 3 and 4 (every
      (bin2, bin1) key, the empty and few-step pixels, the first and last
      pixel of every row band and every chunk) and the reference driver's
      codes and scales for those pixels (minutes on a few cores).
  python tests/golden/make_golden.py refcuda       (on a B200)
      Runs the reference's unmodified driver + CUDA back end
      (oracle/_ref/tessera_encode_cuda_ref, built by `make -C oracle cuda-ref`)
      on the same case tiles: <case>_refcuda.npz. This is the reference's own
      network arithmetic (cuBLASLt, bf16 biases) on the same inputs; it pins
      the CPU restatement, which the test suite compares against it.

Case tiles and weights are regenerated from seeds (tessera-inference_b200/synth.py).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path[:0] = [str(REPO / "tessera-inference_b200"), str(REPO / "oracle")]
import synth  # noqa: E402

# name -> (tile kwargs, weight perturbation)
CASES = {
    "cfg0": (dict(synth.CONFIGS[0]), 0.0),
    "cloudy": (dict(H=32, W=32, T2=60, Ta=30, Td=30, p=0.15, seed=31, cloudy=True), 0.05),
    "long": (dict(H=6, W=8, T2=300, Ta=150, Td=150, p=0.92, seed=32), 0.05),
}


def case_tile(name: str) -> dict:
    return synth.make_tile(**CASES[name][0])


def case_weights(name: str, wdir: Path) -> Path:
    perturb = CASES[name][1]
    return synth.make_weights(wdir / f"w_{perturb}.tcw", seed=0, perturb=perturb)


def numpy_pad_pattern(n: int, B: int) -> np.ndarray:
    if n == 0:
        return np.zeros(B, np.int64)
    if n >= B:
        return np.linspace(0, n - 1, B, dtype=np.int64)
    remain = B - n
    if remain <= n:
        extra = np.array([g[len(g) // 2] for g in np.array_split(np.arange(n), remain)], np.int64)
    else:
        extra = np.arange(remain) % n
    return np.concatenate([np.arange(n), extra]).astype(np.int64)


PAD_N = list(range(0, 41)) + [55, 63, 64, 65, 99, 100, 119, 120, 121, 127, 128, 129, 150, 199, 200, 201,
                              255, 256, 257, 270, 300, 333, 1000]
PAD_B = [1, 2, 3, 5, 8, 16, 24, 32, 40, 64, 72, 120, 128, 200, 248, 256]


def padpattern():
    keys, vals = [], []
    for n in PAD_N:
        for B in PAD_B:
            keys.append((n, B))
            vals.append(numpy_pad_pattern(n, B))
    off = np.cumsum([0] + [len(v) for v in vals]).astype(np.int64)
    np.savez_compressed(HERE / "pad_pattern.npz", nB=np.array(keys, np.int64), off=off,
                        idx=np.concatenate(vals).astype(np.int16))
    print("pad_pattern.npz:", len(keys), "cases")


def read_dump(path: Path):
    b = path.read_bytes()
    G, T2, T1 = struct.unpack_from("<3q", b, 0)
    o = 24
    s2 = np.frombuffer(b, np.float32, G * T2 * 11, o); o += 4 * G * T2 * 11
    s1 = np.frombuffer(b, np.float32, G * T1 * 3, o); o += 4 * G * T1 * 3
    out = np.frombuffer(b, np.float32, G * 128, o)
    return G, T2, T1, s2, s1, out


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def run_driver(binary: Path, name: str, work: Path, dump: bool):
    tile = case_tile(name)
    tdir = synth.write_tile_dir(tile, work / name / f"grid_{name}")
    w = case_weights(name, work)
    out = work / name / "out"
    env = dict(os.environ)
    dd = work / name / "dump"
    if dump:
        dd.mkdir(parents=True, exist_ok=True)
        env["TC_ORACLE_DUMP"] = str(dd)
    subprocess.run([str(binary), str(tdir), str(out), str(w)], check=True, env=env)
    codes = np.load(out / f"grid_{name}.npy")
    scales = np.load(out / f"grid_{name}_scales.npy")
    batches, outs = [], []
    if dump:
        for f in sorted(dd.glob("batch_*.bin")):
            G, T2, T1, s2, s1, o = read_dump(f)
            batches.append({"G": G, "T2": T2, "T1": T1, "s2": sha(s2), "s1": sha(s1)})
            outs.append(np.array(o).reshape(G, 128))
    return codes, scales, batches, outs


def driver():
    binary = REPO / "oracle" / "_ref" / "tessera_encode_ref"
    if not binary.exists():
        sys.exit("build the reference driver first: make -C oracle")
    with tempfile.TemporaryDirectory() as td:
        for name in CASES:
            codes, scales, batches, outs = run_driver(binary, name, Path(td), dump=True)
            extra = {}
            if name == "long":  # the f32 embeddings the driver quantised (pins the quantisation)
                import oracle
                emb = np.zeros((codes.shape[0] * codes.shape[1], 128), np.float32)
                for (pix, _, _), o in zip(oracle.group_batches(case_tile(name)), outs):
                    emb[pix] = o
                extra["emb"] = emb
            np.savez_compressed(HERE / f"{name}_oracle.npz", codes=codes, scales=scales, **extra)
            (HERE / f"{name}_batches.json").write_text(json.dumps(batches, indent=0))
            print(name, codes.shape, len(batches), "batches")


def refcuda():
    binary = REPO / "oracle" / "_ref" / "tessera_encode_cuda_ref"
    if not binary.exists():
        sys.exit("build the reference CUDA driver first: make -C oracle cuda-ref")
    outdir = Path(os.environ.get("GOLDEN_OUT", HERE))
    outdir.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory() as td:
        for name in CASES:
            codes, scales, _, _ = run_driver(binary, name, Path(td), dump=False)
            np.savez_compressed(outdir / f"{name}_refcuda.npz", codes=codes, scales=scales)
            print(name, codes.shape)


# config -> (pixels sampled per (bin2, bin1) key, row-band splits whose band
# and chunk boundaries are covered). Config 4 runs one whole tile per GPU.
SUBSETS = {1: (150, (1, 2, 4, 8)), 3: (150, (1, 2, 4, 8)), 4: (100, (1,))}
# the library's default chunk caps (TC_CHUNK_TOKENS, TC_CHUNK_PIXELS)
CHUNK_TOKENS, CHUNK_PIXELS = 524288, 32768


def chunk_starts(t2: np.ndarray, t1: np.ndarray, tok_cap: int = CHUNK_TOKENS, px_cap: int = CHUNK_PIXELS):
    """First pixel (relative to the band) of every chunk the library's planner
    cuts a band into: each chunk takes pixels while it holds at most px_cap
    pixels and tok_cap tokens of either modality (encode_band in
    tessera-inference_b200/csrc/backend.cu)."""
    o2 = np.concatenate([[0], np.cumsum(t2)])
    o1 = np.concatenate([[0], np.cumsum(t1)])
    n, i0, starts = len(t2), 0, []
    while i0 < n:
        starts.append(i0)
        a = int(np.searchsorted(o2, o2[i0] + tok_cap, side="right")) - 1
        b = int(np.searchsorted(o1, o1[i0] + tok_cap, side="right")) - 1
        i1 = min(n, i0 + px_cap, a, b)
        if i1 <= i0:
            raise ValueError("a pixel larger than the token cap")
        i0 = i1
    return starts


def subset_pixels(cfg: int, tile: dict) -> np.ndarray:
    """The stratified pixel subset of a benchmark configuration: a seeded sample
    of every (bin2, bin1) key present (the pixels with no observation, key 0,
    and the one-modality and few-step keys included), plus the first and last
    pixel of every row band of each split and of every chunk of each band."""
    import oracle
    import tessera_b200 as tb
    per_key, splits = SUBSETS[cfg]
    T2, H, W = tile["masks"].shape
    n2, n1 = oracle.counts(tile)
    key = oracle.bin_size(n2) * 1000 + oracle.bin_size(n1)
    rng = np.random.default_rng(100 + cfg)
    pick = []
    for k in np.unique(key):
        idx = np.flatnonzero(key == k)
        pick.append(rng.choice(idx, size=min(per_key, idx.size), replace=False))
    t2, t1 = oracle.tile_tokens(tile)
    for nb in splits:
        rows = tb.plan_rows(tile, nb) if nb > 1 else [0, H]
        for r0, r1 in zip(rows, rows[1:]):
            p0, p1 = r0 * W, r1 * W
            if p1 <= p0:
                continue
            s = np.array(chunk_starts(t2[p0:p1], t1[p0:p1]), np.int64) + p0
            pick += [s, s[1:] - 1, np.array([p1 - 1], np.int64)]
    return np.unique(np.concatenate(pick)).astype(np.int64)


def subsets(cfgs=(1, 3, 4)):
    """<cfgN>_subset.npz: for configs 1, 3 and 4, the stratified pixel subset
    (subset_pixels) and the codes and scales the reference's unmodified driver
    with the CPU back-end restatement writes for those pixels, run as one 1 x K
    tile (exact: every pixel's result depends only on its own series)."""
    binary = REPO / "oracle" / "_ref" / "tessera_encode_ref"
    if not binary.exists():
        sys.exit("build the reference driver first: make -C oracle")
    with tempfile.TemporaryDirectory() as td:
        w = synth.make_weights(Path(td) / "w.tcw", seed=0)
        for cfg in cfgs:
            tile = synth.make_config_tile(cfg)
            pix = subset_pixels(cfg, tile)
            sub = synth.subset_tile(tile, pix)
            del tile
            tdir = synth.write_tile_dir(sub, Path(td) / f"grid_cfg{cfg}")
            out = Path(td) / "out"
            r = subprocess.run([str(binary), str(tdir), str(out), str(w)], check=True, capture_output=True, text=True)
            codes = np.load(out / f"grid_cfg{cfg}.npy").reshape(-1, 128)
            scales = np.load(out / f"grid_cfg{cfg}_scales.npy").reshape(-1)
            np.savez_compressed(HERE / f"cfg{cfg}_subset.npz", pixels=pix, codes=codes, scales=scales)
            print(f"cfg{cfg}: {pix.size} px;", r.stdout.strip().splitlines()[0])


API_NAMES = ("tc_create", "tc_encode", "tc_profile_dump", "tc_destroy")


def c_prototypes(text: str, names=API_NAMES) -> dict:
    """name -> token list of its declaration `ret name(params);` in C source
    text (comments removed, whitespace ignored)."""
    import re
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    text = re.sub(r"//[^\n]*", " ", text)
    out = {}
    for n in names:
        m = re.search(r"(?:^|[;{}])\s*([A-Za-z_][\w\s\*]*?\b" + n + r"\s*\([^)]*\)\s*;)", text, flags=re.M)
        if m:
            out[n] = re.findall(r"\w+|[^\s\w]", m.group(1))
    return out


def reference_root() -> Path:
    return Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))


def api():
    """ref_api.json: the token lists of the four back-end prototypes the
    reference driver declares (src/tessera_encode.cpp:47-52)."""
    src = reference_root() / "src" / "tessera_encode.cpp"
    if not src.exists():
        sys.exit(f"the reference driver is needed: {src}")
    protos = c_prototypes(src.read_text())
    if set(protos) != set(API_NAMES):
        sys.exit(f"could not find all four prototypes in {src}: {sorted(protos)}")
    (HERE / "ref_api.json").write_text(json.dumps(protos, indent=1) + "\n")
    print({k: " ".join(v) for k, v in protos.items()})


def export():
    import torch
    script = reference_root() / "tools" / "export_weights.py"
    if not script.exists():
        sys.exit(f"the reference's exporter is needed: {script}")
    res = {}
    with tempfile.TemporaryDirectory() as td:
        for dtype in ("float32", "bfloat16"):
            ck = Path(td) / f"ck_{dtype}.pt"
            torch.save(synth.fake_checkpoint(7, dtype), ck)
            out = Path(td) / f"ref_{dtype}.tcw"
            subprocess.run([sys.executable, str(script), str(ck), str(out)], check=True)
            data = out.read_bytes()
            res[dtype] = {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data)}
    (HERE / "export_ref.json").write_text(json.dumps(res, indent=1) + "\n")
    print(res)


if __name__ == "__main__":
    cmd = sys.argv[1] if len(sys.argv) > 1 else "all"
    if cmd in ("padpattern", "all"):
        padpattern()
    if cmd in ("driver", "all"):
        driver()
    if cmd in ("export", "all"):
        export()
    if cmd in ("api", "all"):
        api()
    if cmd == "refcuda":
        refcuda()
    if cmd == "subsets":
        subsets(tuple(int(c) for c in sys.argv[2:]) or (1, 3, 4))
