""".tcw weight files: the tensor list of the v2 Large pixel student, reader,
writer and checker.

Format (the reference's tools/export_weights.py:31-39, kept byte-compatible so
files from either tool load in either back end): b"TCW1", u32 tensor count,
then per tensor u32 name_len, the name, u32 ndim, i64 dims[ndim] and the f32
data, row-major and little-endian.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

D, FF, NL, RED, OUT = 640, 2560, 4, 2560, 128


def weight_shapes() -> list[tuple[str, tuple[int, ...]]]:
    """Every tensor the Large student's C++ back ends read (tessera_cpu.cpp:459-502)."""
    out = []
    for pre, c in (("s2_backbone", 10), ("s1_backbone", 2)):
        out += [(f"{pre}.embedding.0.weight", (D, c)), (f"{pre}.embedding.0.bias", (D,)),
                (f"{pre}.embedding.2.weight", (D, D)), (f"{pre}.embedding.2.bias", (D,))]
        for l in range(NL):
            L = f"{pre}.transformer_encoder.layers.{l}"
            out += [(f"{L}.self_attn.in_proj_weight", (3 * D, D)), (f"{L}.self_attn.in_proj_bias", (3 * D,)),
                    (f"{L}.self_attn.out_proj.weight", (D, D)), (f"{L}.self_attn.out_proj.bias", (D,)),
                    (f"{L}.linear1.weight", (FF, D)), (f"{L}.linear1.bias", (FF,)),
                    (f"{L}.linear2.weight", (D, FF)), (f"{L}.linear2.bias", (D,)),
                    (f"{L}.norm1.weight", (D,)), (f"{L}.norm1.bias", (D,)),
                    (f"{L}.norm2.weight", (D,)), (f"{L}.norm2.bias", (D,))]
        out += [(f"{pre}.attn_pool.query.weight", (1, D)), (f"{pre}.attn_pool.query.bias", (1,))]
    out += [("dim_reducer.0.weight", (RED, 2 * D)), ("dim_reducer.0.bias", (RED,)),
            ("dim_reducer.1.weight", (RED,)), ("dim_reducer.1.bias", (RED,)),
            ("dim_reducer.4.weight", (OUT, RED)), ("dim_reducer.4.bias", (OUT,))]
    return out


def check_large(shapes: dict[str, tuple[int, ...]]) -> list[str]:
    """Problems that would make tc_create reject a file with these tensors:
    a missing tensor or a wrong shape, in the order tc_create checks them
    (its validate_large). Extra tensors are allowed and ignored by the back end."""
    problems = []
    for name, want in weight_shapes():
        got = shapes.get(name)
        if got is None:
            problems.append(f"missing tensor {name}")
        elif tuple(got) != want:
            problems.append(f"{name} has shape {tuple(got)}, expected {want}")
    return problems


def write_tcw(path: Path | str, w: dict[str, np.ndarray]) -> None:
    """Writes the tensors in the dict's order, each converted to f32."""
    with open(path, "wb") as f:
        f.write(b"TCW1")
        f.write(struct.pack("<I", len(w)))
        for k, v in w.items():
            v = np.ascontiguousarray(v, dtype=np.float32)
            name = k.encode()
            f.write(struct.pack("<I", len(name)))
            f.write(name)
            f.write(struct.pack("<I", v.ndim))
            f.write(struct.pack(f"<{v.ndim}q", *v.shape))
            f.write(v.tobytes())


def read_tcw(path: Path | str) -> dict[str, np.ndarray]:
    """Reads every tensor as a read-only f32 view of the file's bytes. Raises
    ValueError on a bad magic number or a truncated file."""
    data = Path(path).read_bytes()
    if data[:4] != b"TCW1" or len(data) < 8:
        raise ValueError(f"{path}: bad weights file")
    (n,) = struct.unpack_from("<I", data, 4)
    o, w = 8, {}
    try:
        for _ in range(n):
            (ln,) = struct.unpack_from("<I", data, o); o += 4
            name = data[o:o + ln].decode(); o += ln
            (nd,) = struct.unpack_from("<I", data, o); o += 4
            shape = struct.unpack_from(f"<{nd}q", data, o); o += 8 * nd
            cnt = int(np.prod(shape)) if nd else 1
            w[name] = np.frombuffer(data, np.float32, cnt, o).reshape(shape); o += 4 * cnt
    except (struct.error, ValueError, UnicodeDecodeError) as e:
        raise ValueError(f"{path}: truncated weights ({e})") from None
    return w
