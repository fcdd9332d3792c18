"""CPU oracle, numpy part: a restatement of the reference driver's pre- and
post-processing (src/tessera_encode.cpp of mtelvers/tessera-inference).

TEST INFRASTRUCTURE ONLY. Nothing in the product imports this module; tests,
`__graft_entry__.smoke()` and bench.py's CPU-baseline leg use it as the checker.

Pinned against: numpy's own linspace / array_split (the functions the
reference's comments say pad_pattern mirrors, src/tessera_encode.cpp:157,169),
and the reference driver itself: oracle/_ref/tessera_encode_ref (the
unmodified src/tessera_encode.cpp linked with the C++ back-end restatement in
oracle/tessera_oracle.cpp) dumps the records it hands to tc_encode, which the
golden fixtures under tests/golden/ hold.
"""
from __future__ import annotations

import numpy as np

# src/tessera_encode.cpp:60-67
S2_MEAN = np.array([1633.0042, 1341.1090, 1539.5536, 3054.8269, 3117.4658,
                    2004.1648, 2694.7275, 2945.1504, 2266.6079, 1657.3094], np.float32)
S2_STD = np.array([1999.4603, 2014.7549, 1929.2201, 1754.2493, 1649.9807,
                   1936.8988, 1748.6041, 1708.6991, 1207.5250, 1108.6046], np.float32)
S1A_MEAN = np.array([5909.3921, 3405.0322], np.float32)
S1A_STD = np.array([1507.1750, 1531.2615], np.float32)
S1D_MEAN = np.array([5816.1382, 3277.7576], np.float32)
S1D_STD = np.array([1554.6475, 1546.4733], np.float32)
EPS = np.float32(1e-9)
EMB = 128


def bin_size(n):
    """src/tessera_encode.cpp:146-151: next multiple of 8 >= n, capped at 256; 0 if n == 0."""
    n = np.asarray(n, np.int64)
    return np.where(n <= 0, 0, np.minimum((n + 7) // 8 * 8, 256)).astype(np.int64)


def pad_pattern(n: int, B: int) -> np.ndarray:
    """src/tessera_encode.cpp:154-180 (_pad_pattern): B indices into [0, n)."""
    out = np.zeros(B, np.int64)
    if n == 0:
        return out
    if n >= B:
        if B == 1:
            return out
        delta, div = float(n - 1), float(B - 1)
        step = delta / div
        for i in range(B):
            y = (float(i) / div) * delta if step == 0 else float(i) * step
            out[i] = int(np.floor(y))
        out[B - 1] = n - 1
        return out
    out[:n] = np.arange(n)
    remain = B - n
    if remain <= n:
        q, r = divmod(n, remain)
        start = 0
        for g in range(remain):
            ln = q + (1 if g < r else 0)
            out[n + g] = start + ln // 2
            start += ln
    else:
        out[n:] = np.arange(remain) % n
    return out


def counts(tile: dict):
    """Per-pixel valid counts, src/tessera_encode.cpp:249-255 (S2 mask != 0,
    S1 either band != 0, ascending and descending summed)."""
    T2, H, W = tile["masks"].shape
    N = H * W
    n2 = (tile["masks"].reshape(T2, N) != 0).sum(0).astype(np.int64)
    n1 = np.zeros(N, np.int64)
    for k in ("asc", "desc"):
        a = tile[k]
        if a.shape[0]:
            n1 += (a.reshape(a.shape[0], N, 2) != 0).any(-1).sum(0)
    return n2, n1


def pixel_records(tile: dict, p: int, b2: int, b1: int):
    """Records one pixel contributes to a tc_encode batch of key (b2, b1),
    src/tessera_encode.cpp:281-329: valid steps first (stable), padded with
    pad_pattern, z-scored in f32. Returns (s2 (B2,11), s1 (B1,3)) f32."""
    T2, H, W = tile["masks"].shape
    N = H * W
    Ta, Td = tile["asc"].shape[0], tile["desc"].shape[0]
    B2, B1 = max(b2, 1), max(b1, 1)
    s2 = np.zeros((B2, 11), np.float32)
    s1 = np.zeros((B1, 3), np.float32)
    if b2 > 0:
        m = tile["masks"].reshape(T2, N)[:, p]
        pos = np.concatenate([np.flatnonzero(m != 0), np.flatnonzero(m == 0)])
        nv = int((m != 0).sum())
        pat = pad_pattern(nv, B2)
        steps = pos[pat]
        src = tile["bands"].reshape(T2, N, 10)[steps, p].astype(np.float32)
        s2[:, :10] = (src - S2_MEAN) / (S2_STD + EPS)
        s2[:, 10] = tile["doys"][steps].astype(np.float32)
    if b1 > 0:
        a = tile["asc"].reshape(Ta, N, 2)[:, p] if Ta else np.zeros((0, 2), np.int16)
        d = tile["desc"].reshape(Td, N, 2)[:, p] if Td else np.zeros((0, 2), np.int16)
        v = np.concatenate([a, d], 0)
        valid = (v != 0).any(-1)
        pos = np.concatenate([np.flatnonzero(valid), np.flatnonzero(~valid)])
        pat = pad_pattern(int(valid.sum()), B1)
        steps = pos[pat]
        for k, s in enumerate(steps):
            if s < Ta:
                s1[k, :2] = (v[s].astype(np.float32) - S1A_MEAN) / (S1A_STD + EPS)
                s1[k, 2] = np.float32(tile["asc_doy"][s])
            else:
                s1[k, :2] = (v[s].astype(np.float32) - S1D_MEAN) / (S1D_STD + EPS)
                s1[k, 2] = np.float32(tile["desc_doy"][s - Ta])
    return s2, s1


def group_batches(tile: dict, batch: int = 4096):
    """The reference's grouping (src/tessera_encode.cpp:258-277): pixels stable-
    sorted by key bin2*1000+bin1, key 0 skipped, each group cut into batches.
    Yields (pixel indices, b2, b1)."""
    n2, n1 = counts(tile)
    key = bin_size(n2) * 1000 + bin_size(n1)
    order = np.argsort(key, kind="stable")
    ks = key[order]
    g0 = 0
    while g0 < len(order):
        g1 = g0
        while g1 < len(order) and ks[g1] == ks[g0]:
            g1 += 1
        b2, b1 = int(ks[g0] // 1000), int(ks[g0] % 1000)
        if not (b2 == 0 and b1 == 0):
            for c0 in range(g0, g1, batch):
                yield order[c0:min(g1, c0 + batch)], b2, b1
        g0 = g1


def quantize(emb: np.ndarray):
    """src/tessera_encode.cpp:344-361: per-pixel scale max(max|e|, 1e-12)/127,
    codes round-half-even(e / scale) clipped to +-127. f32 arithmetic."""
    e = np.asarray(emb, np.float32)
    am = np.maximum(np.abs(e).max(-1), np.float32(1e-12)).astype(np.float32)
    sc = (am / np.float32(127.0)).astype(np.float32)
    q = np.rint(e / sc[..., None])
    q = np.clip(q, -127, 127).astype(np.int8)
    return q, sc


def pixel_flop(t2, t1):
    """Algorithmic FLOP of one pixel with token counts t2, t1 (0, 0 = skipped)."""
    t2 = np.asarray(t2, np.float64)
    t1 = np.asarray(t1, np.float64)
    ftok = lambda c: 1280.0 * c + 819200.0 + 39321600.0
    f = t2 * ftok(10) + t1 * ftok(2) + 10240.0 * (t2 * t2 + t1 * t1) + 7208960.0
    return np.where((t2 == 0) & (t1 == 0), 0.0, f)


def tile_tokens(tile: dict):
    """Per-pixel token counts (max(bin,1) per modality; 0, 0 for a pixel
    with no observation)."""
    n2, n1 = counts(tile)
    b2, b1 = bin_size(n2), bin_size(n1)
    none = (b2 == 0) & (b1 == 0)
    t2 = np.where(none, 0, np.maximum(b2, 1))
    t1 = np.where(none, 0, np.maximum(b1, 1))
    return t2, t1


def compare(ref_codes, ref_scales, codes, scales) -> dict:
    """The metrics of the reference's tools/compare.py:7-22, plus the
    acceptance checks (int8 |diff| <= 1 share, scale relative diff, zero codes)."""
    a = ref_codes.astype(np.int32).reshape(-1, EMB)
    b = codes.astype(np.int32).reshape(-1, EMB)
    sa, sb = ref_scales.reshape(-1), scales.reshape(-1)
    d = np.abs(a - b)
    valid = (sa > 0) & (sb > 0) & np.isfinite(sa) & np.isfinite(sb)
    na, nb = np.linalg.norm(a, axis=-1), np.linalg.norm(b, axis=-1)
    ok = valid & (na > 0) & (nb > 0)
    cos = (a * b).sum(-1)[ok] / (na[ok] * nb[ok]) if ok.any() else np.ones(1)
    rs = np.abs(sa[ok] - sb[ok]) / np.maximum(np.abs(sa[ok]), 1e-12) if ok.any() else np.zeros(1)
    zero_ref = (a == 0).all(-1)
    return {
        "exact": float(np.mean(d == 0)), "off1": float(np.mean(d == 1)), "off2plus": float(np.mean(d >= 2)),
        "max": int(d.max()) if d.size else 0, "within1": float(np.mean(d <= 1)),
        "cos_mean": float(cos.mean()), "cos_p1": float(np.percentile(cos, 1)), "cos_min": float(cos.min()),
        "scale_rel_median": float(np.median(rs)), "scale_rel_p99": float(np.percentile(rs, 99)),
        "scale_rel_max": float(rs.max()),
        "zero_rows_ref": int(zero_ref.sum()),
        "zero_rows_match": bool(np.array_equal(zero_ref, (b == 0).all(-1))),
        "empty_scale_exact": bool(np.array_equal(sa[zero_ref].view(np.uint32), sb[zero_ref].view(np.uint32))),
    }
