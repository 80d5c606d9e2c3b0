"""Parity against the REFERENCE's own CUDA kernels, recompiled for sm_100a from its sources by
oracle/build_ref.py (its mma.sync fused GEMM and its small kernels, with its --use_fast_math flags),
run on the same inputs on the same GPU as this build's kernels.

Known reference behaviour excluded here (and documented): with --use_fast_math the reference's fused
GEMM flushes s_inv = 2^-127 to zero for rows whose max is zero or below 2^-113, then multiplies by
1/0 and returns NaN for those rows; this build keeps the exact subnormal and returns the bias."""
import pathlib

import pytest
import torch

import inputs
from helpers import assert_close_ulp, bits_equal, edge_rows, gemm_tolerance, rel_err

pytestmark = pytest.mark.gpu

REF_DIR = pathlib.Path(__file__).resolve().parents[1] / "oracle" / "_ref"


def _ref(name):
    if not (REF_DIR / f"{name}.so").exists():
        pytest.skip("oracle/_ref not built (needs the reference sources: python oracle/build_ref.py)")
    from oracle.build_ref import load_ref
    return load_ref(name)


@pytest.mark.parametrize("M,K,N", [(256, 1024, 1024), (4096, 3072, 3072), (512, 4096, 4096), (333, 520, 1032)])
def test_linear_vs_reference_fused_kernel(M, K, N):
    from tbf16 import ops
    ref = _ref("tbf16_ref_gemm")
    x = inputs.gemm_x(M, K, seed=5 + M, device="cuda")
    w = inputs.gemm_w(N, K, seed=6 + N, device="cuda")
    b = (torch.randn(N, device="cuda") * 0.1).bfloat16()
    w16, ws = ops.prepare_weight(w)
    y = ops.scaled_linear(x, w16, ws, b)
    y_ref = ref.linear(x, w16, ws, b, -1, 15, False)
    absprod = (x.double().abs() @ w16.double().abs().t()) * ws.double()[None, :]
    # both sides accumulate in fp32 (different orders): twice the accumulation bound
    tol = gemm_tolerance(y_ref.cpu(), 2 * absprod.cpu(), K)
    assert_close_ulp(y.cpu(), y_ref.cpu(), tol, frac_exact=0.9, what=f"vs reference fused {M}x{K}x{N}")
    exact = x.double() @ w.double().t() + b.double()
    assert rel_err(y, exact) < 2e-3 and rel_err(y_ref, exact) < 2e-3


def test_reference_fused_kernel_zero_row_behaviour():
    """Documents the reference's fast-math behaviour on an all-zero row: its s_inv = 2^-127 flushes to 0,
    the kernel converts with 1/0 and the row comes out NaN; this build returns the bias for that row."""
    from tbf16 import ops
    ref = _ref("tbf16_ref_gemm")
    x = inputs.gemm_x(256, 512, seed=1, device="cuda")
    x[3] = 0
    w = inputs.gemm_w(256, 512, seed=2, device="cuda")
    b = (torch.randn(256, device="cuda") * 0.1).bfloat16()
    w16, ws = ops.prepare_weight(w)
    y_ref = ref.linear(x, w16, ws, b, -1, 15, False)
    y = ops.scaled_linear(x, w16, ws, b)
    assert torch.isnan(y_ref[3].float()).all()
    assert torch.equal(y[3], b)
    others = torch.arange(256, device="cuda") != 3
    assert torch.isfinite(y_ref[others].float()).all()


def test_row_scale_vs_reference_kernel():
    ref = _ref("tbf16_ref_gemm")
    from tbf16 import _ext as E
    x = edge_rows(300, 2048, seed=2).cuda()
    s_ref = ref.row_scale(x, 15, False)
    s = torch.empty(300, device="cuda")
    E.call("tbf16_row_scale", E.ptr(x), 300, 2048, 2048, 15, 0, E.ptr(s), None, None, 0, E.stream_ptr())
    amax = torch.nan_to_num(x.float(), nan=0.0).abs().amax(1)  # fmaxf semantics: NaN ignored
    normal = amax >= 2.0 ** -113  # below: the reference flushes s_inv = 2^-127 to 0
    assert torch.equal(s[normal], s_ref[normal])
    assert (s_ref[~normal] == 0).all() and (s[~normal] == 2.0 ** -127).all()


@pytest.mark.parametrize("t", [0, -1, 15])
def test_quantize_rows_vs_reference_kernel(t):
    from tbf16 import ops
    small = _ref("tbf16_ref_small")
    x = edge_rows(200, 1024, seed=7 + t).cuda()
    y, s = ops.quantize_rows(x, t, False)
    y_ref, s_ref = small.quantize_rows(x, t, False)
    # the reference's fast-math s_inv flushes 2^-127 (only reachable with t=15 on zero/tiny rows)
    keep = s_ref != 0
    assert torch.equal(s[keep], s_ref[keep])
    # rows with fp32-subnormal products differ under flush-to-zero: compare rows above that range
    # and rows of bf16-subnormal inputs (the reference's flush-to-zero zeroes them before scaling)
    keep &= torch.nan_to_num(x.float(), nan=0.0).abs().amax(1) >= 2.0 ** -126
    assert bits_equal(y[keep], y_ref[keep])


def test_quantize_cols_vs_reference_kernel():
    small = _ref("tbf16_ref_small")
    from tbf16 import _ext as E
    R, K = 1000, 512
    x = inputs.gemm_x(R, K, seed=3, device="cuda")
    rm = torch.exp2(torch.randint(-6, 7, (R,), device="cuda").float())
    y_ref, s_ref = small.quantize_cols(x, -2, rm)
    y = torch.empty(R, K, device="cuda", dtype=torch.float16)
    s = torch.empty(K, device="cuda")
    ws = torch.empty(K, device="cuda")
    E.call("tbf16_quantize_cols", E.ptr(x), R, K, K, -2, E.ptr(rm), E.ptr(y), K, E.ptr(s), E.ptr(ws), E.stream_ptr())
    assert torch.equal(s, s_ref) and bits_equal(y, y_ref)


def test_head_amax_and_scale_vs_reference_kernel():
    small = _ref("tbf16_ref_small")
    from tbf16 import _ext as E
    q, k, v = inputs.attention_qkv(2, 4, 256, 64, seed=1, device="cuda")
    amax_ref = small.head_amax(q)
    amax = torch.empty(8, device="cuda")
    E.call("tbf16_head_amax", E.ptr(q), E.BF16, 2, 4, 256, 64, *q.stride()[:3], E.ptr(amax), E.stream_ptr())
    assert torch.equal(amax.view(2, 4), amax_ref)
    e = (torch.arange(8, device="cuda", dtype=torch.int32) - 4).view(2, 4).contiguous()
    y_ref = small.head_scale_cast(v, e, torch.float16)
    y = torch.empty_like(y_ref)
    E.call("tbf16_head_scale_cast", E.ptr(v), E.BF16, 2, 4, 256, 64, *v.stride()[:3], E.ptr(e), 4, 1, E.ptr(y), E.F16,
           E.stream_ptr())
    assert bits_equal(y, y_ref)
