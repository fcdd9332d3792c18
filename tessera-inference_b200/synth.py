"""Seeded synthetic stand-ins for the reference's inputs.

The real checkpoint (student_large.pt) and the Manchester tile are not
available, so tests and benchmarks use:

* `make_weights`: Large-architecture weights, Xavier-uniform for every 2-D
  weight, zero biases, LayerNorm weight 1 / bias 0, written in the .tcw format
  of the reference's tools/export_weights.py:31-39 (b"TCW1", u32 count, then
  per tensor u32 name_len, name, u32 ndim, i64 dims, f32 data).
* `make_tile`: staged tiles with the value distributions of the benchmark
  configurations (uint16 S2 bands in 0..10000, Bernoulli masks, sorted days
  of year, int16 S1 backscatter Normal(-1500, 400)), in the array layout the
  reference driver loads (tessera_encode.cpp:182-209, README.md:58-68).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from tcw import read_tcw, weight_shapes, write_tcw  # noqa: F401  (re-exported for tests)


def random_weights(seed: int = 0, perturb: float = 0.0) -> dict[str, np.ndarray]:
    """Xavier-uniform weights, zero biases, unit LayerNorm. perturb > 0 adds
    seeded noise of that scale to every bias and LayerNorm parameter (used to
    exercise the bias and affine paths, which are zero/identity otherwise)."""
    rng = np.random.default_rng(seed)
    w = {}
    for name, shape in weight_shapes():
        is_ln = ".norm" in name or name.startswith("dim_reducer.1.")
        if len(shape) == 2:
            fan_out, fan_in = shape
            bound = np.sqrt(6.0 / (fan_in + fan_out))
            a = rng.uniform(-bound, bound, size=shape)
        elif is_ln and name.endswith(".weight"):
            a = np.ones(shape)
        else:
            a = np.zeros(shape)
        w[name] = a.astype(np.float32)
    if perturb > 0:
        rng2 = np.random.default_rng(seed + 1000)
        for name, shape in weight_shapes():
            if len(shape) == 1:
                w[name] = (w[name] + perturb * rng2.standard_normal(shape)).astype(np.float32)
    return w


def fake_checkpoint(seed: int = 7, dtype: str = "float32", extra: bool = True) -> dict:
    """A stand-in for the training checkpoint that tools/export_weights.py
    reads: {"model": state dict of torch tensors, "args": the Large student's
    sizes}. Values are random_weights(seed, perturb=0.1) in the given torch
    dtype; extra=True adds two tensors the back ends do not read."""
    import torch
    sd = {k: torch.from_numpy(np.array(v)).to(getattr(torch, dtype))
          for k, v in random_weights(seed, perturb=0.1).items()}
    if extra:
        rng = np.random.default_rng(seed + 1)
        sd["s2_backbone.extra_head.weight"] = torch.from_numpy(rng.standard_normal((3, 5)).astype(np.float32)).to(
            getattr(torch, dtype))
        sd["step_count"] = torch.tensor([12345.0])
    args = {"latent_dim": 160, "num_layers": 4, "nhead": 4, "dim_feedforward": 2560, "repr_dim": 128,
            "enable_qk_norm": False, "lr": 1e-4}
    return {"model": sd, "args": args}


def make_weights(path: Path | str, seed: int = 0, perturb: float = 0.0) -> Path:
    path = Path(path)
    if not path.exists():
        tmp = path.with_suffix(path.suffix + ".tmp")
        write_tcw(tmp, random_weights(seed, perturb))
        tmp.replace(path)
    return path


# ---------------------------------------------------------------- tiles
CONFIGS = {
    0: dict(H=64, W=64, T2=40, Ta=20, Td=20, p=0.7, seed=1),
    1: dict(H=1113, W=695, T2=120, Ta=60, Td=60, p=0.6, seed=2),
    3: dict(H=1024, W=1024, T2=120, Ta=60, Td=60, p=0.15, seed=3, cloudy=True),
    4: dict(H=1100, W=1100, T2=250, Ta=120, Td=120, p=0.6, seed=4),
}


def _s1(rng, T, H, W):
    x = np.rint(rng.normal(-1500.0, 400.0, size=(T, H, W, 2)))
    return np.clip(x, -32768, 32767).astype(np.int16)


def make_tile(H: int, W: int, T2: int, Ta: int, Td: int, p: float, seed: int, cloudy: bool = False) -> dict:
    """Synthetic staged tile. cloudy=True adds config 3's edge cases: 5% of
    pixels with no observation at all, 20% with 1-4 valid S2 and S1 steps,
    1% S2-only and 1% S1-only pixels."""
    rng = np.random.default_rng(seed)
    t = {
        "bands": rng.integers(0, 10001, size=(T2, H, W, 10), dtype=np.uint16),
        "masks": (rng.random((T2, H, W), dtype=np.float32) < p).astype(np.uint8),
        "doys": np.sort(rng.integers(1, 366, size=T2)).astype(np.uint16),
        "asc": _s1(rng, Ta, H, W),
        "asc_doy": np.sort(rng.integers(1, 366, size=Ta)).astype(np.int16),
        "desc": _s1(rng, Td, H, W),
        "desc_doy": np.sort(rng.integers(1, 366, size=Td)).astype(np.int16),
    }
    if cloudy:
        N = H * W
        cat = rng.choice(5, size=N, p=[0.05, 0.20, 0.01, 0.01, 0.73])
        m = t["masks"].reshape(T2, N)
        a = t["asc"].reshape(Ta, N, 2)
        d = t["desc"].reshape(Td, N, 2)
        none = np.flatnonzero(cat == 0)
        m[:, none] = 0
        a[:, none] = 0
        d[:, none] = 0
        few = np.flatnonzero(cat == 1)
        if few.size:
            m[:, few] = 0
            k2 = rng.integers(1, 5, size=few.size)
            order = np.argsort(rng.random((few.size, T2), dtype=np.float32), axis=1)
            for j in range(4):
                sel = k2 > j
                m[order[sel, j], few[sel]] = 1
            T1 = Ta + Td
            keep = np.zeros((T1, few.size), bool)
            k1 = rng.integers(1, 5, size=few.size)
            order1 = np.argsort(rng.random((few.size, T1), dtype=np.float32), axis=1)
            for j in range(4):
                sel = k1 > j
                keep[order1[sel, j], np.flatnonzero(sel)] = True
            a[:, few] *= keep[:Ta, :, None]
            d[:, few] *= keep[Ta:, :, None]
        s2only = np.flatnonzero(cat == 2)
        a[:, s2only] = 0
        d[:, s2only] = 0
        s1only = np.flatnonzero(cat == 3)
        m[:, s1only] = 0
    return t


def make_config_tile(cfg: int, **over) -> dict:
    c = dict(CONFIGS[cfg])
    c.update(over)
    return make_tile(**c)


def write_tile_dir(tile: dict, d: Path | str) -> Path:
    """Write a tile in the reference's staged layout (s2/ and s1/ subdirs)."""
    d = Path(d)
    (d / "s2").mkdir(parents=True, exist_ok=True)
    (d / "s1").mkdir(parents=True, exist_ok=True)
    np.save(d / "s2" / "bands.npy", tile["bands"])
    np.save(d / "s2" / "masks.npy", tile["masks"])
    np.save(d / "s2" / "doys.npy", tile["doys"])
    np.save(d / "s1" / "sar_ascending.npy", tile["asc"])
    np.save(d / "s1" / "sar_ascending_doy.npy", tile["asc_doy"])
    np.save(d / "s1" / "sar_descending.npy", tile["desc"])
    np.save(d / "s1" / "sar_descending_doy.npy", tile["desc_doy"])
    return d


def subset_tile(tile: dict, pixels: np.ndarray) -> dict:
    """1 x K tile of the given flat pixel indices (same days of year). Exact for
    parity: each pixel's result depends only on its own series."""
    T2, H, W = tile["masks"].shape
    N = H * W
    K = len(pixels)
    out = dict(tile)
    out["bands"] = np.ascontiguousarray(tile["bands"].reshape(T2, N, 10)[:, pixels].reshape(T2, 1, K, 10))
    out["masks"] = np.ascontiguousarray(tile["masks"].reshape(T2, N)[:, pixels].reshape(T2, 1, K))
    for k in ("asc", "desc"):
        T = tile[k].shape[0]
        out[k] = np.ascontiguousarray(tile[k].reshape(T, N, 2)[:, pixels].reshape(T, 1, K, 2))
    return out
