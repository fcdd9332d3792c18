"""Opt-in kernel variants, each in a subprocess with its environment switch
(the library reads TC_ATTN_TC, TC_LN_FUSE, TC_GEMM_VARIANT and TC_GEMM_TN_PAIR once at load):
whole-tile parity against the oracle golden for the mma.sync attention on
every chunk (TC_ATTN_TC=0), the tcgen05
attention on every chunk of series up to 128 steps, short ones included
(TC_ATTN_TC=2), the single-CTA GEMM on every layer (TC_GEMM_VARIANT=1), the
operand-swapped GEMM on every layer it takes (=3), its CTA-pair form on every
layer without a residual (=4), the per-layer choice with that pair form
(TC_GEMM_TN_PAIR=1), the LayerNorm-fused GEMM epilogue and the CTA-pair
(cta_group::2) GEMM."""
import os
import subprocess
import sys

import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

CODE = r"""
import sys, tempfile
from pathlib import Path
sys.path[:0] = [{pkg!r}, {orc!r}, {tests!r}]
import numpy as np, oracle, tessera_b200 as tb
from golden.make_golden import case_tile, case_weights
from test_gpu_parity import assert_acceptance
g = np.load(Path({tests!r}) / "golden" / "cloudy_oracle.npz")
with tempfile.TemporaryDirectory() as td:
    enc = tb.Encoder(case_weights("cloudy", Path(td)))
    codes, scales = enc.encode_tile(case_tile("cloudy"))
    enc.close()
m = oracle.compare(g["codes"], g["scales"], codes, scales)
print(m)
assert_acceptance(m)
"""


@pytest.mark.parametrize("env", [{"TC_ATTN_TC": "0"}, {"TC_ATTN_TC": "2"}, {"TC_GEMM_VARIANT": "1"},
                                 {"TC_GEMM_VARIANT": "3"}, {"TC_GEMM_VARIANT": "4"}, {"TC_GEMM_TN_PAIR": "1"},
                                 {"TC_LN_FUSE": "1"}, {"TC_GEMM_VARIANT": "2"}])
def test_variant_parity(env):
    code = CODE.format(pkg=str(REPO / "tessera-inference_b200"), orc=str(REPO / "oracle"), tests=str(REPO / "tests"))
    r = subprocess.run([sys.executable, "-c", code], env=dict(os.environ, **env), capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
