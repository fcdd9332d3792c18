"""The tile driver tessera_b200_encode (the reference's command line, tile I/O
pipelined against the GPU): its .npy outputs meet the acceptance tolerance
against the oracle golden, equal the library's own tc_encode_tile bit for bit
when several tiles go through one call, and bad inputs fail with a message."""
import subprocess

import numpy as np
import pytest

import oracle
import synth
import tessera_b200 as tb
from conftest import GOLDEN, REPO
from golden.make_golden import CASES, case_tile, case_weights
from test_gpu_parity import assert_acceptance

pytestmark = pytest.mark.gpu

DRIVER = REPO / "tessera-inference_b200" / "tessera_b200_encode"


def run_driver(tiles, out, weights, env=None):
    import os
    return subprocess.run([str(DRIVER), ",".join(str(t) for t in tiles), str(out), str(weights)], capture_output=True,
                          text=True, env=dict(os.environ, **(env or {})), timeout=600)


@pytest.mark.parametrize("case", list(CASES))
def test_driver_golden(case, tmp_path):
    tdir = synth.write_tile_dir(case_tile(case), tmp_path / f"grid_{case}")
    r = run_driver([tdir], tmp_path / "out", case_weights(case, tmp_path))
    assert r.returncode == 0, r.stderr
    assert f"ENCODE grid=grid_{case}" in r.stdout and "TOTAL tiles=1" in r.stdout
    codes = np.load(tmp_path / "out" / f"grid_{case}.npy")
    scales = np.load(tmp_path / "out" / f"grid_{case}_scales.npy")
    g = np.load(GOLDEN / f"{case}_oracle.npz")
    m = oracle.compare(g["codes"], g["scales"], codes, scales)
    print(case, m)
    assert_acceptance(m)


def test_driver_many_tiles_match_library(tmp_path):
    """Four tiles of three shapes in one call (both pipeline slots reused):
    every output equals tc_encode_tile on the same arrays, bit for bit."""
    tiles = [synth.make_tile(H=24, W=20, T2=30, Ta=12, Td=10, p=0.7, seed=51),
             case_tile("cloudy"),
             synth.make_tile(H=7, W=33, T2=50, Ta=0, Td=25, p=0.5, seed=52),
             synth.make_tile(H=24, W=20, T2=30, Ta=12, Td=10, p=0.4, seed=53)]
    dirs = [synth.write_tile_dir(t, tmp_path / f"t{i}") for i, t in enumerate(tiles)]
    w = case_weights("cloudy", tmp_path)
    r = run_driver(dirs, tmp_path / "out", w)
    assert r.returncode == 0, r.stderr
    assert r.stdout.count("ENCODE grid=") == 4 and "TOTAL tiles=4" in r.stdout
    enc = tb.Encoder(w)
    try:
        for i, t in enumerate(tiles):
            codes, scales = enc.encode_tile(t)
            assert np.array_equal(np.load(tmp_path / "out" / f"t{i}.npy"), codes), i
            assert np.array_equal(np.load(tmp_path / "out" / f"t{i}_scales.npy").view(np.uint32),
                                  scales.view(np.uint32)), i
    finally:
        enc.close()


def test_driver_rejects_wrong_dtype(tmp_path):
    t = synth.make_tile(H=8, W=8, T2=10, Ta=5, Td=5, p=0.7, seed=54)
    d = synth.write_tile_dir(t, tmp_path / "bad")
    np.save(d / "s2" / "masks.npy", t["masks"].astype(np.int16))
    r = run_driver([d], tmp_path / "out", case_weights("cfg0", tmp_path))
    assert r.returncode == 1
    assert "masks.npy: element type <i2, this input must be |u1" in r.stderr
