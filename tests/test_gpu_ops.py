"""Per-kernel parity of the CUDA stages against plain PyTorch fp32 references
that apply the reference's rounding points (bf16 at every layer boundary, f32
accumulation and statistics; src/tessera_cpu.cpp:215-263,333-343,434-455).

Tolerance (written here because it is the contract of these tests): outputs
are bf16 and the reference is rounded to bf16 from an f32 value computed in a
different summation order, so an element may differ by one bf16 ulp
(2^-7 relative at most) plus the f32 accumulation error, bounded here by
2^-17 * sum_k |a_k w_k| (about 7.6e-6 of the magnitude sum). Near-zero results
of cancelling sums can change sign within that bound, which is why a pure ulp
count is not used. At least 95% of elements must also match exactly, which a
wrong tile layout or a wrong epilogue cannot reach.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import tessera_b200 as tb  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    return tb.load_library()


def _p(t):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Distance in bf16 ulps between two bf16 tensors (sign-magnitude aware)."""
    def key(x):
        i = x.contiguous().view(torch.int16).to(torch.int32)
        return torch.where(i < 0, -(i & 0x7FFF), i)
    return (key(a) - key(b)).abs()


def check_bf16(out, ref, mag=None, exact_frac=0.95, rel=2.0 ** -7, acc=2.0 ** -17, atol=1e-30):
    """out, ref: bf16. mag: per-element sum of |terms| of the reference value
    (f32 accumulation-error scale); defaults to |ref|."""
    o, r = out.float(), ref.float()
    m = r.abs() if mag is None else mag
    tol = rel * r.abs() + acc * m + atol
    err = (o - r).abs()
    bad = err > tol
    frac = (ulp_diff(out, ref) == 0).float().mean().item()
    assert not bad.any(), (f"{bad.sum().item()} of {bad.numel()} out of tolerance; worst err "
                           f"{err[bad].max().item()} (exact {frac:.4f})")
    assert frac >= exact_frac, f"exact fraction {frac}"


def close_bf16(out, ref, ulps=2, atol=1e-3):
    """Attention / pooling tolerance: S and P are each rounded to bf16 before
    the next product, so a near-tie may move an output by about one bf16 ulp
    of |v| ~ 1 (atol 1e-2 covers 2^-7) on top of `ulps` relative ulps."""
    o, r = out.float(), ref.float()
    tol = r.abs() * (ulps * 2.0 ** -8) + atol
    bad = (o - r).abs() > tol
    assert not bad.any(), f"{bad.sum().item()} elements out of tolerance; max abs diff {(o - r).abs().max().item()}"


def gemm_ref(A, W, bias, relu, res):
    """(bf16 reference, magnitude sum per element) in fp32 with TF32 off."""
    torch.backends.cuda.matmul.allow_tf32 = False
    y = A.float() @ W.float().t()
    mag = A.float().abs() @ W.float().abs().t()
    if bias is not None:
        y = y + bias
        mag = mag + bias.abs()
    if relu:
        y = torch.relu(y)
    if res is not None:
        y = y + res.float()
        mag = mag + res.float().abs()
    return y.to(torch.bfloat16), mag


GEMM_SHAPES = [
    (1, 640, 640), (127, 1920, 640), (128, 2560, 640), (300, 640, 2560), (333, 2560, 1280),
    (200, 128, 2560), (4096, 1920, 640), (65536, 640, 640), (20000, 2560, 640), (20000, 640, 2560),
]


@pytest.mark.parametrize("variant", [1, 2, 3, 4])
@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("mode", ["bias", "bias_relu", "bias_res"])
def test_gemm(lib, M, N, K, mode, variant):
    """variant 1: single-CTA tiles; 2: CTA pairs; 3: weights on the MMA's M side
    (operand-swapped, transposing epilogue)."""
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16) if mode == "bias_res" else None
    relu = mode == "bias_relu"
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.tcb_op_gemm(_p(A), K, _p(W), _p(bias), int(relu), _p(res), N, None, 1, None, None, _p(out), N,
                         M, N, K, 0, variant, _p(status), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    ref, mag = gemm_ref(A, W, bias, relu, res)
    check_bf16(out, ref, mag)


@pytest.mark.parametrize("variant", [1, 2])
@pytest.mark.parametrize("bn", [128, 160, 256])
def test_gemm_tile_widths(lib, bn, variant):
    M, N, K = 1000, 1280, 640
    g = torch.Generator(device="cuda").manual_seed(bn)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    rc = lib.tcb_op_gemm(_p(A), K, _p(W), None, 0, None, 0, None, 1, None, None, _p(out), N, M, N, K, bn, variant,
                         None, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    ref, mag = gemm_ref(A, W, None, False, None)
    check_bf16(out, ref, mag)


@pytest.mark.parametrize("N,bn", [(1200, 256), (400, 0), (48, 0), (640, 0), (1920, 0), (1200, 160), (208, 128)])
def test_gemm_tail_tile(lib, N, bn):
    """Column tiles of width bn with a narrower last tile (N not a multiple of
    bn), through the residual epilogue: 1200 = 4*256 + 176, 400 = 256 + 144,
    48 = one 48-wide tile, 640 = 256 + 256 + 128, 1200 = 7*160 + 80, 208 = 128 + 80."""
    M, K = 1000, 640
    g = torch.Generator(device="cuda").manual_seed(N + bn)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.tcb_op_gemm(_p(A), K, _p(W), _p(bias), 0, _p(res), N, None, 1, None, None, _p(out), N, M, N, K, bn, 1,
                         _p(status), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    ref, mag = gemm_ref(A, W, bias, False, res)
    check_bf16(out, ref, mag)


def test_gemm_pe_residual(lib):
    """Residual = bf16 day-of-year sinusoid: table rows for integer days in
    [0, 366], sin/cos of doy * div for any other value."""
    M, N, K = 777, 640, 640
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    div = torch.exp(torch.arange(0, 640, 2, dtype=torch.float32) * -(np.log(10000.0) / 640.0)).cuda()
    days = torch.arange(367, dtype=torch.float32, device="cuda")
    ang = days[:, None] * div[None, :]
    table = torch.stack([torch.sin(ang), torch.cos(ang)], -1).reshape(367, 640).to(torch.bfloat16)
    doy = torch.randint(0, 367, (M,), device="cuda", generator=g).float()
    doy[::50] = 12.5  # non-integer: computed, not looked up
    doy[1::50] = 400.0  # out of table range
    rec = torch.zeros(M, 3, device="cuda")
    rec[:, 2] = doy
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    rc = lib.tcb_op_gemm(_p(A), K, _p(W), None, 0, None, 0, _p(rec[:, 2:]), 3, _p(table), _p(div), _p(out), N,
                         M, N, K, 0, 0, None, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    angr = doy[:, None] * div[None, :]
    pe = torch.stack([torch.sin(angr), torch.cos(angr)], -1).reshape(M, 640).to(torch.bfloat16)
    ref, mag = gemm_ref(A, W, None, False, pe)
    check_bf16(out, ref, mag, rel=2.0 ** -6)


def attention_ref(qkv, off):
    out = torch.zeros(qkv.shape[0], 640, dtype=torch.bfloat16, device=qkv.device)
    scale = np.float32(1.0) / np.sqrt(np.float32(160.0))
    for i in range(len(off) - 1):
        a, b = int(off[i]), int(off[i + 1])
        if b <= a:
            continue
        x = qkv[a:b].float()
        for h in range(4):
            q = x[:, h * 160:(h + 1) * 160]
            k = x[:, 640 + h * 160:640 + (h + 1) * 160]
            v = x[:, 1280 + h * 160:1280 + (h + 1) * 160]
            s = ((q @ k.t()) * float(scale)).to(torch.bfloat16).float()
            p = torch.softmax(s, -1).to(torch.bfloat16).float()
            out[a:b, h * 160:(h + 1) * 160] = (p @ v).to(torch.bfloat16)
    return out


@pytest.mark.parametrize("lens", [[1, 7, 16, 17, 33, 120, 256, 0, 5, 80, 255, 64, 8],
                                  [120] * 300 + [0, 3, 128, 1],
                                  [8, 16, 24, 40, 56, 72, 88, 96] * 40])
def test_attention_segments(lib, lens):
    """The 2nd and 3rd cases (series of at most 128 steps, long enough on
    average) run on the tcgen05 kernel, the 1st (series up to 256) on the
    mma.sync kernel. The forced selections are checked in
    tests/test_gpu_variants.py (selected by environment at load)."""
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    M = int(off[-1])
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(M, 1920, device="cuda", generator=g).to(torch.bfloat16)
    att = torch.zeros(M, 640, device="cuda", dtype=torch.bfloat16)
    doff = torch.from_numpy(off).cuda()
    rc = lib.tcb_op_attention(_p(qkv), _p(doff), 0, len(lens), max(lens), _p(att), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    close_bf16(att, attention_ref(qkv, off), ulps=3, atol=1e-2)


def test_attention_tc_stage_reuse(lib):
    """tcgen05 kernel: many more items than CTAs, so both K/V stages and both
    S/P buffers are reused, with empty pixels and every length class of 16
    interleaved, and a 32-row box boundary at T = 32, 64, 96."""
    rng = np.random.default_rng(3)
    lens = (list(rng.integers(64, 129, size=1900)) + list(rng.integers(0, 64, size=100))
            + [32, 64, 96, 128, 31, 33, 1, 0])
    rng.shuffle(lens)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    M = int(off[-1])
    g = torch.Generator(device="cuda").manual_seed(21)
    qkv = torch.randn(M, 1920, device="cuda", generator=g).to(torch.bfloat16)
    att = torch.zeros(M, 640, device="cuda", dtype=torch.bfloat16)
    doff = torch.from_numpy(off).cuda()
    rc = lib.tcb_op_attention(_p(qkv), _p(doff), 0, len(lens), max(lens), _p(att), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    close_bf16(att, attention_ref(qkv, off), ulps=3, atol=1e-2)


def test_attention_uniform(lib):
    T, P = 120, 37
    g = torch.Generator(device="cuda").manual_seed(12)
    qkv = torch.randn(T * P, 1920, device="cuda", generator=g).to(torch.bfloat16)
    att = torch.zeros(T * P, 640, device="cuda", dtype=torch.bfloat16)
    rc = lib.tcb_op_attention(_p(qkv), None, T, P, T, _p(att), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    close_bf16(att, attention_ref(qkv, np.arange(P + 1) * T), ulps=3, atol=1e-2)


@pytest.mark.parametrize("M", [1, 15, 17, 5000])
def test_layernorm640(lib, M):
    g = torch.Generator(device="cuda").manual_seed(13)
    x = (torch.randn(M, 640, device="cuda", generator=g) * 3 + 1).to(torch.bfloat16)
    gam = torch.randn(640, device="cuda", generator=g)
    bet = torch.randn(640, device="cuda", generator=g)
    y = torch.empty_like(x)
    assert lib.tcb_op_layernorm640(_p(x), M, _p(gam), _p(bet), _p(y), _stream()) == 0
    torch.cuda.synchronize()
    xf = x.float()
    ref = torch.nn.functional.layer_norm(xf, (640,), gam, bet, 1e-5).to(torch.bfloat16)
    # (x - mean) cancels: scale the accumulation term by |x| * rstd * |gamma| + |beta|
    rstd = 1.0 / torch.sqrt(xf.var(-1, unbiased=False, keepdim=True) + 1e-5)
    check_bf16(y, ref, xf.abs() * rstd * gam.abs() + bet.abs(), acc=2.0 ** -14)


def test_pool(lib):
    lens = [1, 8, 72, 120, 256, 0, 3]
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    M = int(off[-1])
    g = torch.Generator(device="cuda").manual_seed(14)
    x = torch.randn(M, 640, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(640, device="cuda", generator=g) * 0.05
    qb = 0.3
    fused = torch.full((len(lens), 1280), 7.0, device="cuda", dtype=torch.bfloat16)
    assert lib.tcb_op_pool(_p(x), _p(torch.from_numpy(off).cuda()), 0, len(lens), _p(q), qb, _p(fused), 640,
                           _stream()) == 0
    torch.cuda.synchronize()
    for i in range(len(lens)):
        a, b = int(off[i]), int(off[i + 1])
        if b == a:
            assert (fused[i, 640:].float() == 0).all()
            continue
        xs = x[a:b].float()
        w = torch.softmax(xs @ q + qb, 0)
        ref = (w[:, None] * xs).sum(0).to(torch.bfloat16)
        close_bf16(fused[i, 640:], ref, ulps=2, atol=1e-3)
        assert (fused[i, :640].float() == 7.0).all()


def test_emb1(lib):
    for C_ in (10, 2):
        M = 3001
        g = torch.Generator(device="cuda").manual_seed(15 + C_)
        rec = torch.randn(M, C_ + 1, device="cuda", generator=g)
        w = (torch.randn(640, C_, device="cuda", generator=g) * 0.3).to(torch.bfloat16).float()
        b = torch.randn(640, device="cuda", generator=g) * 0.1
        y = torch.empty(M, 640, device="cuda", dtype=torch.bfloat16)
        w1t = w.t().contiguous()
        assert lib.tcb_op_emb1(C_, _p(rec), M, _p(w1t), _p(b), _p(y), _stream()) == 0
        torch.cuda.synchronize()
        a = rec[:, :C_].to(torch.bfloat16).float()
        ref = torch.relu(a @ w.t() + b).to(torch.bfloat16)
        check_bf16(y, ref, a.abs() @ w.abs().t() + b.abs())


def test_ln_relu2560(lib):
    P = 300
    g = torch.Generator(device="cuda").manual_seed(16)
    r = torch.randn(P, 2560, device="cuda", generator=g).to(torch.bfloat16)
    gam = torch.randn(2560, device="cuda", generator=g)
    bet = torch.randn(2560, device="cuda", generator=g)
    rf = r.float()
    ref = torch.relu(torch.nn.functional.layer_norm(rf, (2560,), gam, bet, 1e-5).to(torch.bfloat16))
    rstd = 1.0 / torch.sqrt(rf.var(-1, unbiased=False, keepdim=True) + 1e-5)
    mag = rf.abs() * rstd * gam.abs() + bet.abs()
    assert lib.tcb_op_ln_relu2560(_p(r), P, _p(gam), _p(bet), _stream()) == 0
    torch.cuda.synchronize()
    check_bf16(r, ref, mag, acc=2.0 ** -14)


def test_out128_and_quant(lib):
    import oracle
    P = 1000
    g = torch.Generator(device="cuda").manual_seed(17)
    r2 = torch.randn(P, 128, device="cuda", generator=g).to(torch.bfloat16)
    empty = torch.zeros(P, dtype=torch.uint8, device="cuda")
    empty[::97] = 1
    out = torch.empty(P, 128, device="cuda")
    codes = torch.empty(P, 128, dtype=torch.int8, device="cuda")
    scales = torch.empty(P, device="cuda")
    assert lib.tcb_op_out128(_p(r2), P, None, _p(out), None, None, _stream()) == 0
    assert lib.tcb_op_out128(_p(r2), P, _p(empty), None, _p(codes), _p(scales), _stream()) == 0
    torch.cuda.synchronize()
    rf = r2.float()
    ref = torch.nn.functional.layer_norm(rf, (128,), eps=1e-5).to(torch.bfloat16)
    rstd = 1.0 / torch.sqrt(rf.var(-1, unbiased=False, keepdim=True) + 1e-5)
    check_bf16(out.to(torch.bfloat16), ref, rf.abs() * rstd, acc=2.0 ** -14)
    # quantisation is bit-exact given the embedding (the f32 output above)
    e = out.cpu().numpy()
    e[empty.cpu().numpy().astype(bool)] = 0
    qc, qs = oracle.quantize(e)
    np.testing.assert_array_equal(codes.cpu().numpy(), qc)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), qs.view(np.uint32))
    assert np.all(scales.cpu().numpy()[::97] == np.float32(1e-12) / np.float32(127.0))


def test_bounded_wait_reports_status(lib):
    """A wait that nothing will ever satisfy ends after its limit with an error
    status instead of a hang; the context remains usable afterwards."""
    import time
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    assert lib.tcb_op_wait_probe(1000, _p(status), _stream()) == 0  # 1 ms limit
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert status.item() == 6
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0  # context still healthy


@pytest.mark.parametrize("M,K", [(1, 640), (129, 640), (5000, 2560), (70000, 640)])
def test_gemm_layernorm_fused(lib, M, K):
    """out-proj + residual + LayerNorm in one kernel (4-CTA cluster, row
    statistics exchanged through distributed shared memory)."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(640, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(640, device="cuda", generator=g) * 0.1
    res = torch.randn(M, 640, device="cuda", generator=g).to(torch.bfloat16)
    gam = 1 + 0.1 * torch.randn(640, device="cuda", generator=g)
    bet = 0.1 * torch.randn(640, device="cuda", generator=g)
    out = torch.full((M, 640), float("nan"), device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.tcb_op_gemm_ln(_p(A), K, _p(W), _p(bias), _p(res), 640, _p(gam), _p(bet), _p(out), 640, M, K,
                            _p(status), _stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    y, _ = gemm_ref(A, W, bias, False, res)
    yf = y.float()
    ref = torch.nn.functional.layer_norm(yf, (640,), gam, bet, 1e-5).to(torch.bfloat16)
    rstd = 1.0 / torch.sqrt(yf.var(-1, unbiased=False, keepdim=True) + 1e-5)
    # y itself may differ from the reference by one bf16 ulp (at most 2^-7 |y|),
    # which LayerNorm scales by rstd * |gamma|: that is the accumulation term here.
    # rel 2^-6: one bf16 ulp of the larger of the two values when they straddle a power of two
    check_bf16(out, ref, yf.abs() * rstd * gam.abs() + bet.abs(), rel=2.0 ** -6, acc=2.0 ** -7, atol=1e-4,
               exact_frac=0.9)


@pytest.mark.parametrize("M,N,K,mode", [(20000, 640, 2560, "res"), (4099, 640, 640, "relu"), (300, 2560, 640, "bias"),
                                        (1, 128, 2560, "bias"), (4099, 640, 640, "res"), (77, 1920, 640, "res"),
                                        (5000, 1920, 640, "relu"), (77, 1920, 640, "bias")])
def test_gemm_swapped_agrees_with_single(lib, M, N, K, mode):
    """The operand-swapped kernel and its CTA-pair form (which runs layers
    without a residual; with one it falls back to the swapped kernel) compute
    every output from the same products in the same k order as the single-CTA
    kernel, so all three are bit-identical (ragged last token tiles and an
    odd number of 128-feature blocks included), and they meet the GEMM
    tolerance."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g) * 0.1
    res = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16) if mode == "res" else None
    outs = []
    for variant in (1, 3, 4):
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
        status = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert lib.tcb_op_gemm(_p(A), K, _p(W), _p(bias), int(mode == "relu"), _p(res), N, None, 1, None, None, _p(out),
                               N, M, N, K, 0, variant, _p(status), _stream()) == 0
        torch.cuda.synchronize()
        assert status.item() == 0
        outs.append(out)
    ref, mag = gemm_ref(A, W, bias, mode == "relu", res)
    check_bf16(outs[0], ref, mag)
    for other in outs[1:]:
        same = (outs[0].view(torch.int16) == other.view(torch.int16)).float().mean().item()
        print("bit-identical fraction", same)
        assert same == 1.0
