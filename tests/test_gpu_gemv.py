"""Parity of the few-row linear (decode path, tbf16_gemv, M <= 8) with the oracle's restatement of the
reference's single-row kernel (small_kernels.cu:107-132): fp32 products of bf16 x and fp16 w, times ws,
plus bias, one bf16 rounding. Elementwise within one bf16 ulp plus the fp32 summation bound
(K * 2^-24 * sum |x w| ws). Up to ops.GEMV_ROWS rows through tbf16.ops, more through the C ABI directly
(scaled_linear sends those to the skinny GEMM)."""
import pytest
import torch

import inputs
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _check(y, x, w16, ws, b):
    ref = orc.gemv_ref(x, w16, ws, b)
    absprod = (x.double().abs() @ w16.double().abs().t()) * ws.double()[None, :]
    tol = orc.bf16_ulp(ref.double()) + x.shape[1] * 2.0 ** -24 * absprod
    d = (y.double() - ref.double()).abs()
    assert (d <= tol).all(), float((d - tol).max())
    assert torch.isfinite(y.float()).all()


@pytest.mark.parametrize("M,K,N,bias", [(1, 4096, 4096, False), (1, 1024, 1000, True), (2, 520, 264, True),
                                        (3, 8192, 1024, False), (5, 72, 33, True), (8, 4096, 4096, True),
                                        (8, 16384, 256, False),
                                        # two-vector form for 1-2 rows up to K = 4096: at the bound, one past
                                        # it (four-vector form), and a second vector only some threads hold
                                        (2, 4096, 1032, True), (2, 4104, 520, False), (1, 2056, 777, True)])
def test_gemv_vs_oracle(M, K, N, bias):
    from tbf16 import ops
    x = inputs.gemm_x(M, K, seed=M + K)
    w = inputs.gemm_w(N, K, seed=N)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(3)) * 0.1).bfloat16() if bias else None
    w16, ws = ops.prepare_weight(w.cuda())
    if M <= ops.GEMV_ROWS:
        y = ops.small_m_linear(x.cuda(), w16, ws, None if b is None else b.cuda()).cpu()
    else:
        y = _gemv_direct(x.cuda(), w16, ws, None if b is None else b.cuda()).cpu()
    assert y.shape == (M, N) and y.dtype == torch.bfloat16
    _check(y, x, w16.cpu(), ws.cpu(), b)


def _gemv_direct(x, w16, ws, b):
    from tbf16 import _ext as E
    M, K = x.shape
    N = w16.shape[0]
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    E.call("tbf16_gemv", E.ptr(x), M, K, x.stride(0), E.ptr(w16), N, w16.stride(0), E.ptr(ws), E.ptr(b), E.ptr(y), N,
           E.stream_ptr(x.device))
    return y


def test_gemv_strided_rows_and_3d_input():
    """Rows with a leading dimension larger than K, and a (B, T, K) input reshaped by scaled_linear."""
    from tbf16 import _ext as E
    from tbf16 import ops
    K, N = 1024, 768
    big = inputs.gemm_x(4, 2 * K, seed=11)
    x = big[:, :K]
    w16, ws = ops.prepare_weight(inputs.gemm_w(N, K, seed=12).cuda())
    xc = big.cuda()[:, :K]
    y = torch.empty(4, N, device="cuda", dtype=torch.bfloat16)
    E.call("tbf16_gemv", E.ptr(xc), 4, K, xc.stride(0), E.ptr(w16), N, w16.stride(0), E.ptr(ws), None, E.ptr(y), N,
           E.stream_ptr(xc.device))
    _check(y.cpu(), x.contiguous(), w16.cpu(), ws.cpu(), None)
    x3 = inputs.gemm_x(6, K, seed=13).reshape(2, 3, K)
    y3 = ops.scaled_linear(x3.cuda(), w16, ws).cpu()
    assert y3.shape == (2, 3, N)
    _check(y3.reshape(6, N), x3.reshape(6, K), w16.cpu(), ws.cpu(), None)


def test_gemv_rejects_too_many_rows():
    from tbf16 import _ext as E
    x = torch.zeros(9, 64, device="cuda", dtype=torch.bfloat16)
    w16 = torch.zeros(32, 64, device="cuda", dtype=torch.float16)
    ws = torch.ones(32, device="cuda")
    y = torch.empty(9, 32, device="cuda", dtype=torch.bfloat16)
    rc = E.lib().tbf16_gemv(E.ptr(x), 9, 64, 64, E.ptr(w16), 32, 64, E.ptr(ws), None, E.ptr(y), 32,
                            E.stream_ptr(x.device))
    assert rc == 6  # TBF16_ERR_UNSUPPORTED


def test_linear_host_matches_device_path():
    """linear_host (pinned host x and y, chunked over three streams) gives the device path's rows: each
    chunk bit-equal to scaled_linear on the same rows, and within the oracle bounds for a short final
    chunk (GEMV for 3 rows)."""
    from helpers import assert_close_ulp, gemm_tolerance
    from tbf16 import ops
    M, K, N = 2 * 1024 + 5, 512, 768
    x = inputs.gemm_x(M, K, seed=21)
    w16, ws = ops.prepare_weight(inputs.gemm_w(N, K, seed=22).cuda())
    b = (torch.randn(N, generator=torch.Generator().manual_seed(23)) * 0.1).bfloat16()
    hx = torch.empty(M, K, dtype=torch.bfloat16, pin_memory=True)
    hx.copy_(x)
    y = ops.linear_host(hx, w16, ws, b.cuda(), chunk_rows=1024)
    torch.cuda.synchronize()
    assert y.shape == (M, N) and not y.is_cuda
    chunks = ops._host_chunks(M, 1024)
    assert len(chunks) > 2 and max(n for _, n in chunks) <= 1024
    xc = x.cuda()
    for r0, n in chunks:
        ref = ops.scaled_linear(xc[r0:r0 + n], w16, ws, b.cuda()).cpu()
        assert torch.equal(y[r0:r0 + n].view(torch.int16), ref.view(torch.int16)), (r0, n)
    w16c, wsc = w16.cpu(), ws.cpu()
    y_ref, _ = orc.linear_fused(x, w16c, wsc, b)
    absprod = (x.double().abs() @ w16c.double().abs().t()) * wsc.double()[None, :]
    assert_close_ulp(y, y_ref, gemm_tolerance(y_ref, absprod, K), what="linear_host")
    y3 = ops.linear_host(hx[:2048 + 3].contiguous(), w16, ws, b.cuda(), chunk_rows=2048)
    torch.cuda.synchronize()
    _check(y3[2048:], x[2048:2051], w16c, wsc, b)
