"""The allocation-free entry point, tcb_op_gemm_ln_noalloc.

Some callers of this library may not allocate device memory: a plugin whose
host framework owns all of the GPU's memory, or a latency-critical path where
cudaMalloc could fail or would stall the device. This entry point takes only
inputs and an output; its scratch is a fixed static device array. The test
calls it through the C ABI twice in a row (the array keeps the first call's
contents, so the second call must not depend on them) and compares each result
with the existing entry point tcb_op_gemm_ln, within the tolerance of the
GEMM + LayerNorm tests; it also checks that a size beyond the array is refused.
This file is collected last so that a failure here cannot hide other tests."""
import pytest

torch = pytest.importorskip("torch")

import tessera_b200 as tb  # noqa: E402

pytestmark = pytest.mark.gpu


def _case(M, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W = (torch.randn(640, K, device="cuda", generator=g) / K ** 0.5).to(torch.bfloat16)
    bias = torch.randn(640, device="cuda", generator=g) * 0.1
    res = torch.randn(M, 640, device="cuda", generator=g).to(torch.bfloat16)
    gam = 1 + 0.1 * torch.randn(640, device="cuda", generator=g)
    bet = 0.1 * torch.randn(640, device="cuda", generator=g)
    return A, W, bias, res, gam, bet


def _both(lib, M, K, seed):
    A, W, bias, res, gam, bet = _case(M, K, seed)
    st = torch.cuda.current_stream().cuda_stream
    ref = torch.full((M, 640), float("nan"), device="cuda", dtype=torch.bfloat16)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.tcb_op_gemm_ln(A.data_ptr(), K, W.data_ptr(), bias.data_ptr(), res.data_ptr(), 640, gam.data_ptr(),
                              bet.data_ptr(), ref.data_ptr(), 640, M, K, status.data_ptr(), st) == 0
    out = torch.full((M, 640), float("nan"), device="cuda", dtype=torch.bfloat16)
    assert lib.tcb_op_gemm_ln_noalloc(A.data_ptr(), K, W.data_ptr(), bias.data_ptr(), res.data_ptr(), 640,
                                      gam.data_ptr(), bet.data_ptr(), out.data_ptr(), M, K, st) == 0
    torch.cuda.synchronize()
    assert status.item() == 0
    # Tolerance of tests/test_gpu_ops.py::test_gemm_layernorm_fused: the two
    # paths may round y differently by one bf16 ulp (LayerNorm scales that by
    # rstd * |gamma|), and outputs may differ by one bf16 ulp.
    y = (A.float() @ W.float().t() + bias + res.float()).to(torch.bfloat16).float()
    rstd = 1.0 / torch.sqrt(y.var(-1, unbiased=False, keepdim=True) + 1e-5)
    mag = y.abs() * rstd * gam.abs() + bet.abs()
    o, r = out.float(), ref.float()
    assert torch.isfinite(o).all()
    tol = 2.0 ** -6 * r.abs() + 2.0 ** -7 * mag + 1e-4
    bad = (o - r).abs() > tol
    assert not bad.any(), f"{bad.sum().item()} elements out of tolerance"
    assert (o == r).float().mean().item() >= 0.9


def test_noalloc_matches_existing_entry_point_twice():
    lib = tb.load_library()
    _both(lib, 8192, 640, 1)   # the largest size the static array holds
    _both(lib, 300, 2560, 2)   # second call, smaller, after the first filled the array


def test_noalloc_rejects_oversize(capfd):
    lib = tb.load_library()
    rc = lib.tcb_op_gemm_ln_noalloc(1, 640, 1, None, None, 640, 1, 1, 1, 8193, 640, None)
    assert rc == -1
    assert "8192" in capfd.readouterr().err


def test_noalloc_after_a_refused_call(capfd):
    """A call the GEMM refuses (K = 100 is not a multiple of 64) returns -1;
    the next valid call starts from a cleared status word and matches the
    existing entry point."""
    lib = tb.load_library()
    A, W, bias, res, gam, bet = _case(64, 640, 3)
    out = torch.empty(64, 640, device="cuda", dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.tcb_op_gemm_ln_noalloc(A.data_ptr(), 100, W.data_ptr(), bias.data_ptr(), res.data_ptr(), 640,
                                    gam.data_ptr(), bet.data_ptr(), out.data_ptr(), 64, 100, st)
    assert rc == -1
    assert "multiple of 64" in capfd.readouterr().err
    _both(lib, 64, 640, 3)
