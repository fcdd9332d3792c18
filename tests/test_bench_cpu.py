"""bench.py's host-side pieces, on the CPU: the parser of the reference
driver's ENCODE timing line (src/tessera_encode.cpp:366-370), the contiguous
row-band sample of the CPU baseline, and the rate summary built from them."""
import importlib.util

import numpy as np

from conftest import REPO

spec = importlib.util.spec_from_file_location("bench", REPO / "bench.py")
bench = importlib.util.module_from_spec(spec)
spec.loader.exec_module(bench)


def test_encode_line_parse():
    line = ("ENCODE grid=grid_sample px=1390 batch_px=4096 batches=9 threads=16  load=0.1s bin=0.0s prep=0.1s "
            "net=14.5s quant+write=0.0s total=14.7s")
    m = bench.ENCODE_RE.search(line)
    assert m is not None
    load, bin_, prep, net, quant, total = (float(x) for x in m.groups())
    assert (load, prep, net, total) == (0.1, 0.1, 14.5, 14.7)


def test_band_pixels_are_contiguous_rows():
    tile = {"masks": np.zeros((3, 10, 7), np.uint8)}
    p = bench.band_pixels(tile, 4, 2)
    np.testing.assert_array_equal(p, np.arange(28, 42))


def test_cpu_summary_rates():
    runs = [{"px": 100, "net_s": 1.0, "total_s": 1.2, "wall_s": 1.25},
            {"px": 300, "net_s": 3.0, "total_s": 3.2, "wall_s": 3.35}]
    sm = bench.cpu_summary(runs)
    assert sm["px"] == 400
    assert abs(sm["net_px_s"] - 100.0) < 1e-9
    assert abs(sm["total_px_s"] - 400 / 4.4) < 1e-9
    assert abs(sm["fixed_cost_frac"] - (4.6 - 4.0) / 4.6) < 1e-9
