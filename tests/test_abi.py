"""C-ABI checks that need no GPU: the library loads, exports every symbol the
public headers declare, rejects bad weight files before touching CUDA, and
plans FLOP-balanced row bands (the multi-GPU sharding) on the host."""
import ctypes as C
import re
import struct

import numpy as np
import pytest

import oracle
import synth
import tessera_b200 as tb
from conftest import REPO


def declared_functions():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(t[a-z]+_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_reference_api():
    names = declared_functions()
    for n in ("tc_create", "tc_encode", "tc_profile_dump", "tc_destroy"):
        assert n in names
    assert len(names) >= 20


def test_reference_prototypes_token_for_token():
    """The four back-end prototypes of include/tessera_b200.h are the ones the
    reference driver declares (src/tessera_encode.cpp:47-52), token for token:
    return type, name, parameter types and names. The reference's tokens are
    the committed fixture tests/golden/ref_api.json (make_golden.py api); when
    the reference tree is on this machine it is read directly as well."""
    import json
    import os
    from pathlib import Path
    from golden.make_golden import API_NAMES, c_prototypes
    ours = c_prototypes((REPO / "include" / "tessera_b200.h").read_text())
    want = json.loads((REPO / "tests" / "golden" / "ref_api.json").read_text())
    assert set(want) == set(API_NAMES)
    for n in API_NAMES:
        assert ours.get(n) == want[n], (n, ours.get(n), want[n])
    src = Path(os.environ.get("REFERENCE_ROOT", "/root/reference")) / "src" / "tessera_encode.cpp"
    if src.exists():
        assert c_prototypes(src.read_text()) == ours


def test_library_exports_every_declared_symbol():
    lib = tb.load_library()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared_functions()) == set(tb.EXPORTED)


def test_weights_rejected_before_cuda(tmp_path, capfd):
    lib = tb.load_library()
    bad = tmp_path / "bad.tcw"
    bad.write_bytes(b"NOPE")
    assert not lib.tc_create(str(bad).encode(), 4)
    assert "is not a .tcw weight file" in capfd.readouterr().err
    assert not lib.tc_create(str(tmp_path / "missing.tcw").encode(), 4)
    assert "cannot open" in capfd.readouterr().err
    # a well-formed file with a wrong shape names the tensor
    w = synth.random_weights(0)
    w["s2_backbone.embedding.2.weight"] = np.zeros((640, 639), np.float32)
    p = tmp_path / "shape.tcw"
    synth.write_tcw(p, w)
    assert not lib.tc_create(str(p).encode(), 4)
    assert "s2_backbone.embedding.2.weight" in capfd.readouterr().err
    # truncated file
    good = tmp_path / "good.tcw"
    synth.write_tcw(good, synth.random_weights(0))
    (tmp_path / "trunc.tcw").write_bytes(good.read_bytes()[:1000])
    assert not lib.tc_create(str(tmp_path / "trunc.tcw").encode(), 4)
    assert "weight file ends at byte 1000" in capfd.readouterr().err
    # bytes after the last tensor
    (tmp_path / "tail.tcw").write_bytes(good.read_bytes() + b"xx")
    assert not lib.tc_create(str(tmp_path / "tail.tcw").encode(), 4)
    assert "2 stray bytes after the last tensor" in capfd.readouterr().err
    w = synth.random_weights(0)
    del w["dim_reducer.4.bias"]
    synth.write_tcw(tmp_path / "miss.tcw", w)
    assert not lib.tc_create(str(tmp_path / "miss.tcw").encode(), 4)
    assert "missing tensor dim_reducer.4.bias" in capfd.readouterr().err


def test_null_handle_errors(capfd):
    lib = tb.load_library()
    assert lib.tc_encode(None, None, 1, 8, None, 8, None) == -1
    assert lib.tc_encode_tile(None, *([None] * 7), 1, 1, 1, 1, 1, None, None) == -1
    lib.tc_destroy(None)
    lib.tc_profile_dump(None)


def test_tcw_roundtrip(tmp_path):
    w = synth.random_weights(0, perturb=0.1)
    p = tmp_path / "w.tcw"
    synth.write_tcw(p, w)
    r = synth.read_tcw(p)
    assert list(r) == list(w)
    for k in w:
        np.testing.assert_array_equal(r[k], w[k])
    b = p.read_bytes()
    assert b[:4] == b"TCW1" and struct.unpack_from("<I", b, 4)[0] == 114


def host_plan_reference(tile, nparts):
    """Same rule as tc_plan_rows, in numpy: cut where the running FLOP sum
    first reaches k/nparts of the total."""
    T2, H, W = tile["masks"].shape
    t2, t1 = oracle.tile_tokens(tile)
    rows = oracle.pixel_flop(t2, t1).reshape(H, W).sum(1)
    total, acc, k = rows.sum(), 0.0, 1
    b = [0] + [H] * nparts
    for r in range(H):
        acc += rows[r]
        while k < nparts and acc >= total * k / nparts:
            b[k] = r + 1
            k += 1
    return b, rows


@pytest.mark.parametrize("nparts", [1, 2, 3, 4, 8])
def test_plan_rows_balanced(nparts):
    tile = synth.make_tile(H=40, W=16, T2=30, Ta=12, Td=12, p=0.5, seed=41, cloudy=True)
    b = tb.plan_rows(tile, nparts)
    ref, rows = host_plan_reference(tile, nparts)
    assert b == ref
    assert b[0] == 0 and b[-1] == 40 and all(x <= y for x, y in zip(b, b[1:]))
    share = [rows[b[i]:b[i + 1]].sum() for i in range(nparts)]
    # each cut lands within one row of its target
    assert max(share) - min(share) <= 2 * rows.max() + 1e-6 * rows.sum()


def test_plan_rows_more_parts_than_rows():
    tile = synth.make_tile(H=3, W=5, T2=8, Ta=4, Td=4, p=0.5, seed=42)
    b = tb.plan_rows(tile, 8)
    assert b[0] == 0 and b[-1] == 3 and len(b) == 9
    assert all(x <= y for x, y in zip(b, b[1:]))


DRIVER = REPO / "tessera-inference_b200" / "tessera_b200_encode"


def test_tile_driver_cli_without_gpu(tmp_path):
    """The tile driver (reference command line) prints its usage on missing
    arguments and fails cleanly, naming the problem, on a bad weights file."""
    import subprocess
    assert DRIVER.exists(), "make -C tessera-inference_b200 builds tessera_b200_encode"
    r = subprocess.run([str(DRIVER)], capture_output=True, text=True)
    assert r.returncode == 2 and "usage:" in r.stderr
    bad = tmp_path / "bad.tcw"
    bad.write_bytes(b"NOPE")
    r = subprocess.run([str(DRIVER), str(tmp_path / "tile"), str(tmp_path / "out"), str(bad)], capture_output=True,
                       text=True)
    assert r.returncode == 1 and "tc_create:" in r.stderr and "is not a .tcw weight file" in r.stderr


def test_host_alloc_rejects_nonpositive():
    lib = tb.load_library()
    assert lib.tc_host_alloc(0) is None
    assert lib.tc_host_alloc(-5) is None
    lib.tc_host_free(None)


def test_attention_classes_follow_each_pixel_alone():
    """Every pixel's attention kernel follows its own series length (bins of
    the reference driver: 1 for an empty modality, multiples of 8 up to 256,
    0 for a pixel with no token), so a pixel's result cannot depend on the
    chunk, row band or device it shares with other pixels."""
    rng = np.random.default_rng(5)
    lens = rng.choice([0, 1, 8, 40, 48, 56, 64, 120, 128, 136, 200, 256], size=500)
    off = np.concatenate([[0], np.cumsum(lens)])
    classes, tmax = tb.attention_plan(off)
    want = [np.flatnonzero((lens > 0) & (lens <= 48)), np.flatnonzero((lens > 48) & (lens <= 128)),
            np.flatnonzero(lens > 128)]
    for c in range(3):
        np.testing.assert_array_equal(classes[c], want[c])
        assert tmax[c] == (int(lens[want[c]].max()) if len(want[c]) else 0)
    # any sub-range (a chunk or row band) puts each pixel in the same class
    for a, b in ((0, 37), (37, 38), (100, 499)):
        sub, _ = tb.attention_plan(off[a:b + 1] - off[a])
        for c in range(3):
            np.testing.assert_array_equal(sub[c] + a, want[c][(want[c] >= a) & (want[c] < b)])
    empty, t0 = tb.attention_plan(np.zeros(1, np.int64))
    assert all(len(x) == 0 for x in empty) and t0 == [0, 0, 0]
    lib = tb.load_library()
    bad = np.array([0, 5, 3], np.int64)
    out = np.zeros(4, np.int64)
    assert lib.tcb_attention_plan(tb._ptr(bad), 2, tb._ptr(np.zeros(2, np.int32)), tb._ptr(out),
                                  tb._ptr(np.zeros(3, np.int32))) == -1



@pytest.mark.parametrize("mode,want_small,want_tc", [("0", lambda t: t <= 128, lambda t: False),
                                                     ("2", lambda t: False, lambda t: t <= 128)])
def test_attention_classes_forced_modes(mode, want_small, want_tc):
    """TC_ATTN_TC=0 sends every series of up to 128 steps to mma.sync, =2 to
    tcgen05; longer series always stay on mma.sync (the mode is read once per
    process, so each runs in its own)."""
    import json
    import os
    import subprocess
    import sys
    code = ("import sys, json, numpy as np; sys.path[:0] = [sys.argv[1]]; import tessera_b200 as tb; "
            "lens = np.array([1, 8, 48, 56, 128, 136, 256, 0]); off = np.concatenate([[0], np.cumsum(lens)]); "
            "c, t = tb.attention_plan(off); print(json.dumps([x.tolist() for x in c]))")
    env = dict(os.environ, TC_ATTN_TC=mode)
    r = subprocess.run([sys.executable, "-c", code, str(REPO / "tessera-inference_b200")], capture_output=True,
                       text=True, env=env, check=True)
    classes = json.loads(r.stdout.strip().splitlines()[-1])
    lens = [1, 8, 48, 56, 128, 136, 256, 0]
    assert classes[0] == [i for i, t in enumerate(lens) if t > 0 and want_small(t)]
    assert classes[1] == [i for i, t in enumerate(lens) if t > 0 and want_tc(t)]
    assert classes[2] == [i for i, t in enumerate(lens) if t > 128]
