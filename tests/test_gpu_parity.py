"""Whole-tile parity of the B200 back end against the CPU oracle through the C ABI.

Acceptance: int8 codes within +-1 on >= 99.9% of elements; all-zero codes
exactly where the reference emits them, with the empty-pixel scale 1e-12f/127
bit-exact; per-pixel scales within 1e-2 relative at the 99th percentile (the
statistic the reference's tools/compare.py:21-22 reports) and within 2^-6
(two bf16 ulps of the largest element) for every pixel. The per-pixel maximum
cannot be held to 1e-2: the scale is max|e|/127 of bf16 values, so one ulp of
a maximum near 2.0 is 0.78% and two are 1.56%; the reference's own CUDA back
end differs from its CPU path by 1.04% (cfg0) and 1.28% (cloudy) on the same
inputs (tests/test_oracle.py::test_oracle_vs_reference_cuda).
The oracle outputs are golden fixtures produced by the reference's own driver
(tests/golden/make_golden.py driver); tiles and weights are regenerated from
their seeds.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
import tessera_b200 as tb  # noqa: E402
from conftest import GOLDEN  # noqa: E402
from golden.make_golden import CASES, case_tile, case_weights  # noqa: E402

pytestmark = pytest.mark.gpu


def assert_acceptance(m: dict):
    assert m["within1"] >= 0.999, m
    assert m["scale_rel_p99"] <= 1e-2, m
    assert m["scale_rel_max"] <= 2.0 ** -6, m
    assert m["zero_rows_match"], m
    assert m["empty_scale_exact"], m


@pytest.mark.parametrize("case", list(CASES))
def test_tile_vs_oracle(case, tmp_path):
    g = np.load(GOLDEN / f"{case}_oracle.npz")
    tile = case_tile(case)
    enc = tb.Encoder(case_weights(case, tmp_path))
    try:
        codes, scales = enc.encode_tile(tile)
    finally:
        enc.close()
    m = oracle.compare(g["codes"], g["scales"], codes, scales)
    print(case, m)
    assert_acceptance(m)


def test_multi_device_handle_matches_single(tmp_path):
    """Row sharding over every visible GPU is byte-identical to one GPU."""
    n = torch.cuda.device_count()
    tile = case_tile("cloudy")
    w = case_weights("cloudy", tmp_path)
    one = tb.Encoder(w)
    c1, s1 = one.encode_tile(tile)
    one.close()
    many = tb.Encoder(w, devices=list(range(n)) * (2 if n == 1 else 1))
    cm, sm = many.encode_tile(tile)
    many.close()
    np.testing.assert_array_equal(cm, c1)
    np.testing.assert_array_equal(sm.view(np.uint32), s1.view(np.uint32))
