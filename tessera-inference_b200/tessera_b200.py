"""ctypes binding of libtessera_b200.so (the C ABI in include/tessera_b200.h and
include/tessera_b200_ops.h).

This is a thin host-side mirror for tests and benchmarks. The product is the
shared library itself, called from C/C++ (the reference driver links it as a
drop-in back end). Loading fails loudly when the library has not been built:
there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libtessera_b200.so"

EXPORTED = [
    "tc_create", "tc_encode", "tc_profile_dump", "tc_destroy",
    "tc_create_multi", "tc_encode_tile", "tc_encode_tile_rows", "tc_encode_tile_device",
    "tc_plan_rows", "tc_set_stream", "tc_set_profiling", "tc_get_stats", "tc_reset_stats", "tc_host_alloc",
    "tc_host_free",
    "tcb_op_gemm", "tcb_op_gemm_ln", "tcb_op_gemm_ln_noalloc", "tcb_op_count", "tcb_op_gather", "tcb_op_emb1", "tcb_op_attention",
    "tcb_op_layernorm640", "tcb_op_pool", "tcb_op_ln_relu2560", "tcb_op_out128", "tcb_op_wait_probe", "tcb_attention_plan",
]

CAT_NAMES = ["h2d", "prep", "emb1", "gemm", "attention", "layernorm", "pool", "head", "d2h"]
GEMM_KINDS = ["emb2", "qkv", "out", "ffn1", "ffn2", "head"]


class TcStats(C.Structure):
    _fields_ = [
        ("calls", C.c_double), ("pixels", C.c_double), ("tokens", C.c_double),
        ("alg_flop", C.c_double), ("gemm_flop", C.c_double), ("gemm_launches", C.c_double),
        ("launches", C.c_double), ("ms_cat", C.c_double * len(CAT_NAMES)),
        ("gemm_ms_kind", C.c_double * 6), ("gemm_flop_kind", C.c_double * 6),
    ]

    def as_dict(self) -> dict:
        d = {k: getattr(self, k) for k, _ in self._fields_ if k not in ("ms_cat", "gemm_ms_kind", "gemm_flop_kind")}
        d["ms_cat"] = {n: self.ms_cat[i] for i, n in enumerate(CAT_NAMES)}
        d["gemm_kind"] = {n: {"ms": self.gemm_ms_kind[i], "flop": self.gemm_flop_kind[i]}
                          for i, n in enumerate(GEMM_KINDS)}
        return d


_lib = None

vp, i64, i32, f32p = C.c_void_p, C.c_int64, C.c_int, C.POINTER(C.c_float)


def load_library(path: os.PathLike | None = None) -> C.CDLL:
    """Load the shared library (built by `make` in this directory)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `make -C {PKG_DIR}` (no fallback exists)")
    lib = C.CDLL(str(p))
    lib.tc_create.restype = vp
    lib.tc_create.argtypes = [C.c_char_p, i32]
    lib.tc_create_multi.restype = vp
    lib.tc_create_multi.argtypes = [C.c_char_p, C.POINTER(C.c_int), i32]
    lib.tc_encode.restype = i32
    lib.tc_encode.argtypes = [vp, vp, i64, i64, vp, i64, vp]
    lib.tc_profile_dump.restype = None
    lib.tc_profile_dump.argtypes = [vp]
    lib.tc_destroy.restype = None
    lib.tc_destroy.argtypes = [vp]
    tile_args = [vp] * 7 + [i64] * 5
    lib.tc_encode_tile.restype = i32
    lib.tc_encode_tile.argtypes = [vp] + tile_args + [vp, vp]
    lib.tc_encode_tile_rows.restype = i32
    lib.tc_encode_tile_rows.argtypes = [vp] + tile_args + [i64, i64, vp, vp]
    lib.tc_encode_tile_device.restype = i32
    lib.tc_encode_tile_device.argtypes = [vp] + tile_args + [i64, i64, vp, vp]
    lib.tc_plan_rows.restype = i32
    lib.tc_plan_rows.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i32, vp]
    lib.tc_set_stream.restype = i32
    lib.tc_set_stream.argtypes = [vp, vp]
    lib.tc_host_alloc.restype = vp
    lib.tc_host_alloc.argtypes = [i64]
    lib.tc_host_free.restype = None
    lib.tc_host_free.argtypes = [vp]
    lib.tc_set_profiling.restype = i32
    lib.tc_set_profiling.argtypes = [vp, i32]
    lib.tc_get_stats.restype = i32
    lib.tc_get_stats.argtypes = [vp, C.POINTER(TcStats)]
    lib.tc_reset_stats.restype = None
    lib.tc_reset_stats.argtypes = [vp]
    lib.tcb_op_gemm.restype = i32
    lib.tcb_op_gemm.argtypes = [vp, i32, vp, vp, i32, vp, i32, vp, i32, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]
    lib.tcb_op_gemm_ln.restype = i32
    lib.tcb_op_gemm_ln.argtypes = [vp, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, i32, vp, vp]
    lib.tcb_op_gemm_ln_noalloc.restype = i32
    lib.tcb_op_gemm_ln_noalloc.argtypes = [vp, i32, vp, vp, vp, i32, vp, vp, vp, i32, i32, vp]
    lib.tcb_op_count.restype = i32
    lib.tcb_op_count.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, vp, vp, vp]
    lib.tcb_op_gather.restype = i32
    lib.tcb_op_gather.argtypes = [i32] + [vp] * 7 + [i64] * 6 + [vp, vp, vp, vp]
    lib.tcb_op_emb1.restype = i32
    lib.tcb_op_emb1.argtypes = [i32, vp, i64, vp, vp, vp, vp]
    lib.tcb_op_attention.restype = i32
    lib.tcb_op_attention.argtypes = [vp, vp, i64, i64, i32, vp, vp]
    lib.tcb_op_layernorm640.restype = i32
    lib.tcb_op_layernorm640.argtypes = [vp, i64, vp, vp, vp, vp]
    lib.tcb_op_pool.restype = i32
    lib.tcb_op_pool.argtypes = [vp, vp, i64, i64, vp, C.c_float, vp, i32, vp]
    lib.tcb_op_ln_relu2560.restype = i32
    lib.tcb_op_ln_relu2560.argtypes = [vp, i64, vp, vp, vp]
    lib.tcb_op_wait_probe.restype = i32
    lib.tcb_op_wait_probe.argtypes = [i64, vp, vp]
    lib.tcb_attention_plan.restype = i32
    lib.tcb_attention_plan.argtypes = [vp, i64, vp, vp, vp]
    lib.tcb_op_out128.restype = i32
    lib.tcb_op_out128.argtypes = [vp, i64, vp, vp, vp, vp, vp]
    if path is None:
        _lib = lib
    return lib


def _ptr(a) -> int | None:
    """Address of a numpy array or torch tensor (None passes NULL)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        assert a.flags["C_CONTIGUOUS"], "arrays must be C-contiguous"
        return a.ctypes.data
    return a.data_ptr()


class Encoder:
    """Handle over tc_create / tc_create_multi with numpy-friendly calls."""

    def __init__(self, weights: os.PathLike, devices: list[int] | None = None):
        self.lib = load_library()
        w = str(weights).encode()
        if devices is None:
            self.h = self.lib.tc_create(w, 4)
        else:
            arr = (C.c_int * len(devices))(*devices)
            self.h = self.lib.tc_create_multi(w, arr, len(devices))
        if not self.h:
            raise RuntimeError("tc_create failed (see stderr)")

    def close(self):
        if self.h:
            self.lib.tc_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, s2: np.ndarray, s1: np.ndarray) -> np.ndarray:
        """tc_encode on prepared (G,T2,11) / (G,T1,3) f32 inputs -> (G,128) f32."""
        s2 = np.ascontiguousarray(s2, dtype=np.float32)
        s1 = np.ascontiguousarray(s1, dtype=np.float32)
        G, T2, _ = s2.shape
        T1 = s1.shape[1]
        out = np.zeros((G, 128), np.float32)
        rc = self.lib.tc_encode(self.h, _ptr(s2), G, T2, _ptr(s1), T1, _ptr(out))
        if rc != 0:
            raise RuntimeError("tc_encode failed")
        return out

    def encode_tile(self, tile: dict, row0: int = 0, row1: int | None = None, codes=None, scales=None):
        """tc_encode_tile_rows on host arrays -> (codes (H,W,128) i8, scales (H,W) f32)."""
        T2, H, W = tile["masks"].shape
        Ta, Td = tile["asc"].shape[0], tile["desc"].shape[0]
        row1 = H if row1 is None else row1
        if codes is None:
            codes = np.zeros((H, W, 128), np.int8)
        if scales is None:
            scales = np.zeros((H, W), np.float32)
        rc = self.lib.tc_encode_tile_rows(
            self.h, _ptr(tile["bands"]), _ptr(tile["masks"]), _ptr(tile["doys"]),
            _ptr(tile["asc"]) if Ta else None, _ptr(tile["asc_doy"]) if Ta else None,
            _ptr(tile["desc"]) if Td else None, _ptr(tile["desc_doy"]) if Td else None,
            T2, Ta, Td, H, W, row0, row1, _ptr(codes), _ptr(scales))
        if rc != 0:
            raise RuntimeError("tc_encode_tile failed")
        return codes, scales

    def encode_tile_device(self, dev: dict, T2, Ta, Td, H, W, row0, row1, codes, scales):
        """tc_encode_tile_device on device-resident tensors (torch)."""
        rc = self.lib.tc_encode_tile_device(
            self.h, _ptr(dev["bands"]), _ptr(dev["masks"]), _ptr(dev["doys"]),
            _ptr(dev.get("asc")), _ptr(dev.get("asc_doy")), _ptr(dev.get("desc")), _ptr(dev.get("desc_doy")),
            T2, Ta, Td, H, W, row0, row1, _ptr(codes), _ptr(scales))
        if rc != 0:
            raise RuntimeError("tc_encode_tile_device failed")

    def set_stream(self, stream_ptr: int | None):
        if self.lib.tc_set_stream(self.h, stream_ptr) != 0:
            raise RuntimeError("tc_set_stream failed")

    def set_profiling(self, on: bool):
        self.lib.tc_set_profiling(self.h, 1 if on else 0)

    def stats(self) -> dict:
        s = TcStats()
        self.lib.tc_get_stats(self.h, C.byref(s))
        return s.as_dict()

    def reset_stats(self):
        self.lib.tc_reset_stats(self.h)

    def profile_dump(self):
        self.lib.tc_profile_dump(self.h)


def attention_plan(off: np.ndarray) -> tuple[list[np.ndarray], list[int]]:
    """tcb_attention_plan: the pixels of each attention class (0: mma.sync,
    1: tcgen05, 2: mma.sync for T > 128) and each class's longest series."""
    lib = load_library()
    off = np.ascontiguousarray(off, dtype=np.int64)
    npix = len(off) - 1
    lst = np.zeros(max(npix, 1), np.int32)
    n = np.zeros(3, np.int64)
    tmax = np.zeros(3, np.int32)
    if lib.tcb_attention_plan(_ptr(off), npix, _ptr(lst), _ptr(n), _ptr(tmax)) != 0:
        raise RuntimeError("tcb_attention_plan failed")
    b = np.concatenate([[0], np.cumsum(n)])
    return [lst[b[c]:b[c + 1]].copy() for c in range(3)], [int(t) for t in tmax]


def plan_rows(tile: dict, nparts: int) -> list[int]:
    """tc_plan_rows: FLOP-balanced contiguous row bands."""
    lib = load_library()
    T2, H, W = tile["masks"].shape
    Ta, Td = tile["asc"].shape[0], tile["desc"].shape[0]
    out = np.zeros(nparts + 1, np.int64)
    rc = lib.tc_plan_rows(_ptr(tile["masks"]), _ptr(tile["asc"]) if Ta else None, _ptr(tile["desc"]) if Td else None,
                          T2, Ta, Td, H, W, nparts, _ptr(out))
    if rc != 0:
        raise RuntimeError("tc_plan_rows failed")
    return [int(x) for x in out]
