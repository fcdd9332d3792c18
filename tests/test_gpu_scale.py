"""Parity at the benchmarked scale.

1. Many chunks on the golden tiles: the library cuts each modality's token
   stream into chunks (TC_CHUNK_TOKENS tokens, TC_CHUNK_PIXELS pixels, read at
   tc_create). With tiny caps (2,048 tokens, 37 pixels: hundreds of chunks, no
   cap a divisor of anything) every golden tile still meets the acceptance
   tolerance against the oracle and is byte-identical to the default-chunk
   output, so chunk offsets (the stream base, the per-chunk attention class
   lists, the output slice) are exercised at every i0 > 0.
2. The full-size tiles of configs 1, 3 and 4 (773,535 / 1,048,576 / 1,210,000
   pixels, hundreds of chunks) encoded whole on the GPU with the default
   chunking, compared on a stratified pixel subset with the reference driver's
   own output for those pixels (tests/golden/cfg{1,3,4}_subset.npz, made by
   make_golden.py subsets): every (bin2, bin1) key, the pixels with no
   observation, and the first and last pixel of every chunk and every 2-, 4-
   and 8-way row band. This replaces the reference's per-key batch loop
   (src/tessera_encode.cpp:266-342) on the tile sizes the benchmark runs.
3. Config 1 split into the 8 FLOP-balanced row bands of an 8-GPU run, each
   band encoded alone (its own chunking), is byte-identical to the whole-tile
   encode on every pixel.
"""
import numpy as np
import pytest

import oracle
import synth
import tessera_b200 as tb
from conftest import GOLDEN
from golden.make_golden import CASES, case_tile, case_weights
from test_gpu_parity import assert_acceptance

pytestmark = pytest.mark.gpu


def encode_with_caps(monkeypatch, weights, tile, tokens, pixels):
    monkeypatch.setenv("TC_CHUNK_TOKENS", str(tokens))
    monkeypatch.setenv("TC_CHUNK_PIXELS", str(pixels))
    enc = tb.Encoder(weights)
    try:
        return enc.encode_tile(tile)
    finally:
        enc.close()
        monkeypatch.delenv("TC_CHUNK_TOKENS")
        monkeypatch.delenv("TC_CHUNK_PIXELS")


@pytest.mark.parametrize("case", list(CASES))
def test_many_chunks_match_oracle_and_default(case, tmp_path, monkeypatch):
    g = np.load(GOLDEN / f"{case}_oracle.npz")
    tile = case_tile(case)
    w = case_weights(case, tmp_path)
    small_c, small_s = encode_with_caps(monkeypatch, w, tile, 2048, 37)
    m = oracle.compare(g["codes"], g["scales"], small_c, small_s)
    print(case, m)
    assert_acceptance(m)
    enc = tb.Encoder(w)
    try:
        c, s = enc.encode_tile(tile)
    finally:
        enc.close()
    np.testing.assert_array_equal(small_c, c)
    np.testing.assert_array_equal(small_s.view(np.uint32), s.view(np.uint32))


@pytest.fixture(scope="module")
def full_encoder(weights_path):
    enc = tb.Encoder(weights_path)
    yield enc
    enc.close()


@pytest.mark.parametrize("cfg", [1, 3, 4])
def test_full_tile_subset_vs_reference(cfg, full_encoder):
    g = np.load(GOLDEN / f"cfg{cfg}_subset.npz")
    tile = synth.make_config_tile(cfg)
    T2, H, W = tile["masks"].shape
    codes, scales = full_encoder.encode_tile(tile)
    pix = g["pixels"]
    m = oracle.compare(g["codes"], g["scales"], codes.reshape(-1, 128)[pix], scales.reshape(-1)[pix])
    print(f"cfg{cfg} ({pix.size} of {H * W} px)", m)
    assert_acceptance(m)
    if cfg == 1:
        bounds = tb.plan_rows(tile, 8)
        bc = np.zeros_like(codes)
        bs = np.zeros_like(scales)
        for r0, r1 in zip(bounds, bounds[1:]):
            full_encoder.encode_tile(tile, r0, r1, bc, bs)
        np.testing.assert_array_equal(bc, codes)
        np.testing.assert_array_equal(bs.view(np.uint32), scales.view(np.uint32))
