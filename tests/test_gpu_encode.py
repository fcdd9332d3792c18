"""Whole-path GPU tests through the C ABI.

1. The tile entry point (device prep + network + quantisation) against the
   reference-API entry point tc_encode fed with records prepared by the numpy
   restatement of the reference driver: bit-identical, because each pixel's
   result depends only on its own records and every kernel is deterministic
   per row/pixel.
2. Edge cases of the reference: pixels with no observation (all-zero codes,
   scale exactly 1e-12f/127), one empty modality (T = 1, zero record), few
   valid steps (array_split and modulo padding), and the error convention.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
import synth  # noqa: E402
import tessera_b200 as tb  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def enc(weights_perturbed_path):
    e = tb.Encoder(weights_perturbed_path)
    yield e
    e.close()


def records_path(enc, tile):
    """Reference-driver batching + tc_encode, then the driver's quantisation."""
    T2, H, W = tile["masks"].shape
    emb = np.zeros((H * W, 128), np.float32)
    for pix, b2, b1 in oracle.group_batches(tile, batch=512):
        recs = [oracle.pixel_records(tile, int(p), b2, b1) for p in pix]
        s2 = np.stack([r[0] for r in recs])
        s1 = np.stack([r[1] for r in recs])
        emb[pix] = enc.encode(s2, s1)
    return oracle.quantize(emb)


@pytest.mark.parametrize("kind", ["plain", "cloudy"])
def test_tile_matches_records_path(enc, kind):
    if kind == "plain":
        tile = synth.make_tile(H=12, W=20, T2=40, Ta=20, Td=20, p=0.7, seed=21)
    else:
        tile = synth.make_tile(H=24, W=24, T2=60, Ta=30, Td=30, p=0.15, seed=22, cloudy=True)
    codes, scales = enc.encode_tile(tile)
    rc, rs = records_path(enc, tile)
    H, W = tile["masks"].shape[1:]
    np.testing.assert_array_equal(codes.reshape(H * W, 128), rc)
    np.testing.assert_array_equal(scales.reshape(-1).view(np.uint32), rs.view(np.uint32))


def test_empty_pixels(enc):
    tile = synth.make_tile(H=8, W=8, T2=16, Ta=8, Td=8, p=0.6, seed=23)
    N = 64
    m = tile["masks"].reshape(16, N)
    a = tile["asc"].reshape(8, N, 2)
    d = tile["desc"].reshape(8, N, 2)
    m[:, [0, 5, 63]] = 0
    a[:, [0, 5, 63]] = 0
    d[:, [0, 5, 63]] = 0
    m[:, 7] = 0          # S1 only
    a[:, 9] = 0          # S2 only
    d[:, 9] = 0
    codes, scales = enc.encode_tile(tile)
    c = codes.reshape(N, 128)
    s = scales.reshape(N)
    for p in (0, 5, 63):
        assert (c[p] == 0).all()
        assert s[p].view(np.uint32) == (np.float32(1e-12) / np.float32(127.0)).view(np.uint32)
    for p in (7, 9):
        assert (c[p] != 0).any()
        assert np.abs(c[p]).max() == 127


def test_row_ranges_compose(enc):
    tile = synth.make_tile(H=10, W=9, T2=24, Ta=12, Td=12, p=0.5, seed=24)
    full_c, full_s = enc.encode_tile(tile)
    c = np.zeros_like(full_c)
    s = np.zeros_like(full_s)
    for r0, r1 in ((0, 3), (3, 4), (4, 10)):
        enc.encode_tile(tile, r0, r1, c, s)
    np.testing.assert_array_equal(c, full_c)
    np.testing.assert_array_equal(s.view(np.uint32), full_s.view(np.uint32))


def test_device_resident_matches_host(enc):
    tile = synth.make_tile(H=16, W=16, T2=30, Ta=15, Td=15, p=0.6, seed=25)
    hc, hs = enc.encode_tile(tile)
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in tile.items()}
    codes = torch.zeros((16, 16, 128), dtype=torch.int8, device="cuda")
    scales = torch.zeros((16, 16), dtype=torch.float32, device="cuda")
    enc.encode_tile_device(dev, 30, 15, 15, 16, 16, 0, 16, codes, scales)
    np.testing.assert_array_equal(codes.cpu().numpy(), hc)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), hs.view(np.uint32))


def test_encode_errors(enc):
    s2 = np.zeros((2, 300, 11), np.float32)
    s1 = np.zeros((2, 8, 3), np.float32)
    with pytest.raises(RuntimeError):
        enc.encode(s2, s1)  # T2 > 256 is rejected, not silently truncated
    assert enc.lib.tc_encode(enc.h, None, 0, 8, None, 8, None) == 0  # G = 0 is a no-op
