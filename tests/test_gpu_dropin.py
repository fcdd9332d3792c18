"""Drop-in check: the reference's own, unmodified driver (src/tessera_encode.cpp)
linked against libtessera_b200.so instead of its CPU or CUDA back end
(oracle/_ref/tessera_encode_b200, `make -C oracle b200-driver`), run on the
golden case tiles, writes .npy outputs that meet the acceptance tolerance
against the oracle golden. It exercises tc_create / tc_encode /
tc_profile_dump / tc_destroy exactly as the reference calls them: batches of at
most TC_BATCH pixels sharing one (T2, T1), in the driver's key order.
"""
import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
import synth
from conftest import GOLDEN, REPO
from golden.make_golden import CASES, case_tile, case_weights
from test_gpu_parity import assert_acceptance

pytestmark = pytest.mark.gpu

DRIVER = REPO / "oracle" / "_ref" / "tessera_encode_b200"


@pytest.mark.parametrize("case", list(CASES))
def test_reference_driver_on_b200(case, tmp_path):
    if not DRIVER.exists():
        pytest.skip("reference driver linked against the B200 back end not built (make -C oracle b200-driver)")
    tdir = synth.write_tile_dir(case_tile(case), tmp_path / f"grid_{case}")
    out = tmp_path / "out"
    r = subprocess.run([str(DRIVER), str(tdir), str(out), str(case_weights(case, tmp_path))], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
    assert "ENCODE grid=" in r.stdout and "TCPROF b200" in r.stdout
    codes = np.load(out / f"grid_{case}.npy")
    scales = np.load(out / f"grid_{case}_scales.npy")
    g = np.load(GOLDEN / f"{case}_oracle.npz")
    m = oracle.compare(g["codes"], g["scales"], codes, scales)
    print(case, m)
    assert_acceptance(m)
