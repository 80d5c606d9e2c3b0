"""Parity of the tcgen05 scaled GEMM with the oracle (gemm_sm75.cu semantics, fp64 accumulation):
elementwise within 1 bf16 ulp plus the fp32-accumulation bound, and within 2e-3 of fp64 including
rows whose magnitudes overflow plain fp16. Called through tbf16.ops (ctypes -> C ABI)."""
import math

import pytest
import torch

import inputs
from helpers import assert_close_ulp, edge_rows, gemm_tolerance, rel_err
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _linear_case(x, w, b, rows=None):
    from tbf16 import ops
    xc, wc = x.cuda(), w.cuda()
    w16, ws = ops.prepare_weight(wc)
    y = ops.scaled_linear(xc, w16, ws, None if b is None else b.cuda()).cpu()
    w16c, wsc = w16.cpu(), ws.cpu()
    sel = torch.arange(x.shape[0]) if rows is None else rows
    xs = x[sel].contiguous()
    y_ref, _ = orc.linear_fused(xs, w16c, wsc, b)
    absprod = (xs.double().abs() @ w16c.double().abs().t()) * wsc.double()[None, :]
    return y[sel], y_ref, absprod, xs, w16c, wsc


@pytest.mark.parametrize("M,K,N,bias", [(256, 1024, 1024, True), (1, 4096, 4096, False), (7, 1024, 512, True),
                                        (130, 4104, 264, True), (333, 520, 1032, False), (64, 64, 256, True),
                                        (512, 2048, 768, False), (1000, 128, 4096, True), (600, 264, 1000, True),
                                        (777, 1024, 520, False)])
def test_linear_vs_oracle(M, K, N, bias):
    x = inputs.gemm_x(M, K, seed=M + K)
    w = inputs.gemm_w(N, K, seed=N + 1)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(3)) * 0.1).bfloat16() if bias else None
    y, y_ref, absprod, xs, w16, ws = _linear_case(x, w, b)
    assert_close_ulp(y, y_ref, gemm_tolerance(y_ref, absprod, K), what=f"linear {M}x{K}x{N}")
    exact = x.double() @ w.double().t() + (b.double() if bias else 0)
    assert rel_err(y, exact) < 2e-3


def test_config1_linear():
    x, w, b = inputs.config1()
    y, y_ref, absprod, *_ = _linear_case(x, w, b)
    assert_close_ulp(y, y_ref, gemm_tolerance(y_ref, absprod, 1024), what="config1")
    over = (x.double().abs().amax(1) > 65504)
    assert over.any()  # rows that overflow plain fp16 are part of the case
    exact = x.double() @ w.double().t() + b.double()
    assert rel_err(y[over], exact[over]) < 2e-3 and rel_err(y, exact) < 2e-3
    assert torch.isfinite(y.float()).all()


def test_linear_edge_rows():
    M, K, N = 160, 256, 512
    x = edge_rows(M, K, seed=4)
    w = inputs.gemm_w(N, K, seed=5)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(6)) * 0.1).bfloat16()
    y, y_ref, absprod, *_ = _linear_case(x, w, b)
    fin = torch.isfinite(x.float()).all(1)
    assert_close_ulp(y[fin], y_ref[fin], gemm_tolerance(y_ref[fin], absprod[fin], K), what="edge rows")
    assert torch.equal(y[0], b)  # an all-zero row gives exactly the bias (no NaN from a flushed scale)
    assert not torch.isfinite(y[6].float()).all() and not torch.isfinite(y[7].float()).all()


@pytest.mark.parametrize("M,K,N", [(8192, 8192, 8192), (4096, 4096, 4096), (16384, 4096, 4096)])
def test_linear_large_sampled(M, K, N):
    """Full-size config-2 shapes: every output finite, sampled rows against the oracle and fp64."""
    from tbf16 import ops
    x = inputs.gemm_x(M, K, seed=11, device="cuda")
    w = inputs.gemm_w(N, K, seed=12, device="cuda")
    w16, ws = ops.prepare_weight(w)
    y = ops.scaled_linear(x, w16, ws)
    assert torch.isfinite(y.float()).all()
    rows = torch.randperm(M, generator=torch.Generator().manual_seed(0))[:48]
    xs = x[rows.cuda()].cpu().contiguous()
    y_ref, _ = orc.linear_fused(xs, w16.cpu(), ws.cpu())
    absprod = (xs.double().abs() @ w16.cpu().double().abs().t()) * ws.cpu().double()[None, :]
    assert_close_ulp(y[rows.cuda()].cpu(), y_ref, gemm_tolerance(y_ref, absprod, K), what=f"{M}x{K}x{N} sampled")
    exact = xs.double() @ w.cpu().double().t()
    assert rel_err(y[rows.cuda()], exact) < 2e-3


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(256, 512, 192), (200, 136, 1000), (640, 520, 192)])
def test_gemm_f16_majors(a_mn, b_mn, M, N, K):
    from tbf16 import ops
    g = torch.Generator().manual_seed(M + N + K + 2 * a_mn + b_mn)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    B = (torch.rand(N, K, generator=g) * 2 - 1).half()
    sa = torch.exp2(torch.randint(-20, 20, (M,), generator=g).float())
    sb = torch.exp2(torch.randint(-20, 20, (N,), generator=g).float())
    bias = (torch.randn(N, generator=g)).bfloat16()
    a_store = A.t().contiguous() if a_mn else A
    b_store = B.t().contiguous() if b_mn else B
    y = ops._gemm_f16(a_store.cuda(), a_mn, b_store.cuda(), b_mn, M, N, K, sa.cuda(), sb.cuda(), bias.cuda()).cpu()
    y_ref = orc.gemm_f16(a_store, a_mn, b_store, b_mn, M, N, K, sa, sb, bias)
    absprod = (A.double().abs() @ B.double().abs().t()) * sa.double()[:, None] * sb.double()[None, :]
    assert_close_ulp(y, y_ref, gemm_tolerance(y_ref, absprod, K), what=f"gemm a_mn={a_mn} b_mn={b_mn}")


def test_linear_q_matches_linear():
    """linear_q on pre-quantised rows and the fused linear agree when given the same fp16 operand."""
    from tbf16 import ops
    x = inputs.gemm_x(300, 1024, seed=21).cuda()
    w = inputs.gemm_w(512, 1024, seed=22).cuda()
    w16, ws = ops.prepare_weight(w)
    x16, sx = ops.quantize_rows(x, 15, False)
    y_q = ops.linear_q(x16, sx, w16, ws)
    exact = x.double() @ w.double().t()
    assert rel_err(y_q, exact) < 2e-3


@pytest.mark.parametrize("M,K,N,bias", [(9, 4096, 4096, True), (16, 8192, 8192, False), (100, 520, 264, True),
                                        (129, 64, 1000, False), (256, 2048, 768, True), (33, 4104, 1032, True),
                                        (200, 1000, 136, False)])
def test_skinny_linear_vs_oracle(M, K, N, bias):
    """9 <= M <= 256 runs the split-K skinny GEMM (weight rows on the MMA's 128-row side, K split over a
    cluster of up to 8 CTAs, partials reduced through distributed shared memory): uneven K splits, a
    single K block, N tails, M padded to 16 columns, all within the oracle bound; two runs bit-equal."""
    from tbf16 import ops
    x = inputs.gemm_x(M, K, seed=M * 7 + K)
    w = inputs.gemm_w(N, K, seed=N + 3)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(5)) * 0.1).bfloat16() if bias else None
    y, y_ref, absprod, *_ = _linear_case(x, w, b)
    assert_close_ulp(y, y_ref, gemm_tolerance(y_ref, absprod, K), what=f"skinny {M}x{K}x{N}")
    w16, ws = ops.prepare_weight(w.cuda())
    y2 = ops.scaled_linear(x.cuda(), w16, ws, None if b is None else b.cuda()).cpu()
    assert torch.equal(y.view(torch.int16), y2.view(torch.int16))


# Products whose last wave of 256-wide pair tiles would leave most CTA pairs idle take other pair tile
# widths: 2048 x 3072 -> 192 columns, 600 x 1000 and 520 x 520 -> 128 (M and N tails, the last tile partly
# past N); 2048 x 2560 (Gemma's o_proj / down_proj at 2048 tokens), 2000 x 2504 (M and N tails) and 1800 x
# 2392 (the last tile's second 160 columns wholly past N: both CTAs' second boxes are zero fill) fit one
# wave of 320-wide tiles (two N = 160 MMAs per k16 step into one accumulator, each CTA's B rows loaded as
# two boxes).
@pytest.mark.parametrize("M,K,N,bias,rows", [(2048, 1024, 3072, True, 64), (2048, 2048, 2560, False, 64),
                                             (2000, 1032, 2504, True, 64), (1800, 520, 2392, False, None),
                                             (600, 1032, 1000, True, None), (520, 256, 520, False, None)])
def test_narrow_pair_tiles_vs_oracle(M, K, N, bias, rows):
    x = inputs.gemm_x(M, K, seed=M + N)
    w = inputs.gemm_w(N, K, seed=K + 3)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(2)) * 0.1).bfloat16() if bias else None
    sel = None if rows is None else torch.randperm(M, generator=torch.Generator().manual_seed(4))[:rows]
    y, y_ref, absprod, xs, w16, ws = _linear_case(x, w, b, sel)
    assert_close_ulp(y, y_ref, gemm_tolerance(y_ref, absprod, K), what=f"narrow tiles {M}x{K}x{N}")
    exact = xs.double() @ w.double().t() + (b.double() if bias else 0)
    assert rel_err(y, exact) < 2e-3
