"""CPU tests of the oracle against golden vectors (no GPU).

* pad_pattern and bin_size against numpy's own linspace / array_split.
* The numpy restatement of the driver's grouping, padding and standardisation
  against the reference driver itself: sha256 of every tc_encode batch the
  unmodified src/tessera_encode.cpp prepared (tests/golden/*_batches.json).
* The numpy quantisation against the codes and scales the reference driver
  wrote from the same embeddings (bit-exact).
* The C++ back-end restatement (oracle/_build/libtessera_oracle.so) against
  the golden outputs the reference driver produced with it, and against the
  reference's own CUDA back end (tests/golden/*_refcuda.npz) within the
  acceptance tolerance, which pins the restatement's network arithmetic.
"""
import ctypes as C
import hashlib
import json
import subprocess
import sys

import numpy as np
import pytest

import oracle
import synth
from conftest import GOLDEN, ORACLE
from golden.make_golden import CASES, case_tile, case_weights

ORACLE_LIB = ORACLE / "_build" / "libtessera_oracle.so"


def test_bin_size_known_answers():
    n = np.array([0, 1, 7, 8, 9, 16, 17, 120, 249, 255, 256, 257, 300, 10000, -3])
    want = np.array([0, 8, 8, 8, 16, 16, 24, 120, 256, 256, 256, 256, 256, 256, 0])
    np.testing.assert_array_equal(oracle.bin_size(n), want)


def test_pad_pattern_vs_numpy_golden():
    g = np.load(GOLDEN / "pad_pattern.npz")
    for i, (n, B) in enumerate(g["nB"]):
        want = g["idx"][g["off"][i]:g["off"][i + 1]].astype(np.int64)
        got = oracle.pad_pattern(int(n), int(B))
        np.testing.assert_array_equal(got, want, err_msg=f"n={n} B={B}")
        if n > 0:
            assert got.max() < n and got.min() >= 0


@pytest.mark.parametrize("case", list(CASES))
def test_prep_matches_reference_driver(case):
    """Every batch the reference driver handed to tc_encode (key order, batch
    cut, valid-first order, pad pattern, z-score bits) is reproduced."""
    golden = json.loads((GOLDEN / f"{case}_batches.json").read_text())
    tile = case_tile(case)
    got = []
    for pix, b2, b1 in oracle.group_batches(tile):
        recs = [oracle.pixel_records(tile, int(p), b2, b1) for p in pix]
        s2 = np.ascontiguousarray(np.stack([r[0] for r in recs]))
        s1 = np.ascontiguousarray(np.stack([r[1] for r in recs]))
        got.append({"G": len(pix), "T2": s2.shape[1], "T1": s1.shape[1],
                    "s2": hashlib.sha256(s2.tobytes()).hexdigest(), "s1": hashlib.sha256(s1.tobytes()).hexdigest()})
    assert got == golden


def test_quantize_matches_reference_driver():
    g = np.load(GOLDEN / "long_oracle.npz")
    codes, scales = oracle.quantize(g["emb"])
    np.testing.assert_array_equal(codes, g["codes"].reshape(-1, 128))
    np.testing.assert_array_equal(scales.view(np.uint32), g["scales"].reshape(-1).view(np.uint32))


def test_empty_pixels_in_reference_output():
    """The reference emits zero codes and scale 1e-12f/127 for pixels with no
    observation; the cloudy golden has such pixels."""
    g = np.load(GOLDEN / "cloudy_oracle.npz")
    t2, t1 = oracle.tile_tokens(case_tile("cloudy"))
    empty = (t2 == 0).reshape(g["scales"].shape)
    assert empty.sum() > 10
    assert (g["codes"][empty] == 0).all()
    assert (g["scales"][empty] == np.float32(1e-12) / np.float32(127.0)).all()
    assert (np.abs(g["codes"][~empty]).max(-1) == 127).all()


def test_pixel_flop_matches_survey_expectation():
    """Config 0 expectation from binomial bins: about 2.905e9 FLOP per pixel."""
    t2, t1 = oracle.tile_tokens(case_tile("cfg0"))
    f = oracle.pixel_flop(t2, t1).mean()
    assert 2.80e9 < f < 3.0e9


@pytest.fixture(scope="module")
def olib():
    if not ORACLE_LIB.exists():
        subprocess.run(["make", "-C", str(ORACLE), "_build/libtessera_oracle.so"], check=True)
    lib = C.CDLL(str(ORACLE_LIB))
    lib.tc_create.restype = C.c_void_p
    lib.tc_create.argtypes = [C.c_char_p, C.c_int]
    lib.tc_encode.restype = C.c_int
    lib.tc_encode.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int64, C.c_void_p]
    lib.tc_destroy.argtypes = [C.c_void_p]
    return lib


def test_oracle_lib_reproduces_golden_subset(olib, tmp_path):
    """A few batches of the 'long' case (T = 256, linspace padding) re-run
    through the C++ restatement give the golden codes bit-exactly."""
    case = "long"
    tile = case_tile(case)
    h = olib.tc_create(str(case_weights(case, tmp_path)).encode(), 4)
    assert h
    g = np.load(GOLDEN / f"{case}_oracle.npz")
    try:
        pix, b2, b1 = next(oracle.group_batches(tile))
        pix = pix[:6]
        recs = [oracle.pixel_records(tile, int(p), b2, b1) for p in pix]
        s2 = np.ascontiguousarray(np.stack([r[0] for r in recs]))
        s1 = np.ascontiguousarray(np.stack([r[1] for r in recs]))
        out = np.zeros((len(pix), 128), np.float32)
        assert olib.tc_encode(h, s2.ctypes.data, len(pix), s2.shape[1], s1.ctypes.data, s1.shape[1],
                              out.ctypes.data) == 0
    finally:
        olib.tc_destroy(h)
    np.testing.assert_array_equal(out.view(np.uint32), g["emb"][pix].view(np.uint32))


def test_oracle_bad_weights(olib, tmp_path):
    p = tmp_path / "bad.tcw"
    p.write_bytes(b"TCW2\x00\x00\x00\x00")
    assert not olib.tc_create(str(p).encode(), 4)


@pytest.mark.parametrize("case", list(CASES))
def test_oracle_vs_reference_cuda(case):
    """Pin of the restatement: the reference's own CUDA back end, run on a
    B200 on the same tile and weights, agrees with the oracle within the
    acceptance tolerance. With zero biases (cfg0) the two compute the same
    function; with non-zero biases the reference CUDA back end rounds them to
    bf16 (src/tessera_cuda.cu:19-20,305,315), a documented difference, so the
    int8 agreement there is held to 99.8%."""
    f = GOLDEN / f"{case}_refcuda.npz"
    if not f.exists():
        pytest.skip("reference CUDA golden not generated yet")
    o = np.load(GOLDEN / f"{case}_oracle.npz")
    r = np.load(f)
    m = oracle.compare(o["codes"], o["scales"], r["codes"], r["scales"])
    print(case, m)
    assert m["within1"] >= (0.999 if CASES[case][1] == 0 else 0.998), m
    assert m["scale_rel_p99"] <= 1e-2, m
    assert m["scale_rel_max"] <= 2.0 ** -6, m
    assert m["cos_min"] >= 0.999, m
    assert m["zero_rows_match"] and m["empty_scale_exact"], m


def test_fp8_study_rounding_matches_torch():
    """The e4m3 rounding of the oracle's FP8 accuracy study (oracle/fp8_study.py)
    is torch's float8_e4m3fn conversion with saturation at 448."""
    import ctypes as C
    torch = pytest.importorskip("torch")
    from conftest import ORACLE
    lib = C.CDLL(str(ORACLE / "_build" / "libtessera_oracle.so"))
    lib.tc_oracle_e4m3.restype = C.c_float
    lib.tc_oracle_e4m3.argtypes = [C.c_float]
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.standard_normal(4000) * np.exp(rng.uniform(-12, 7, 4000)),
                         [0.0, 448, 449, 464, 479, 480, 1000, -1000, 2 ** -9, 2 ** -10, 3 * 2 ** -10, 2 ** -6,
                          1.0625, 1.1875, 232, 248]]).astype(np.float32)
    ours = np.array([lib.tc_oracle_e4m3(float(x)) for x in xs], np.float32)
    ref = torch.from_numpy(xs).clamp(-448, 448).to(torch.float8_e4m3fn).to(torch.float32).numpy()
    np.testing.assert_array_equal(ours, ref)
