"""Parity against the REFERENCE's own CUDA kernels, recompiled for sm_100a from its sources by
oracle/build_ref.py (its mma.sync fused GEMM and its small kernels, with its --use_fast_math flags),
run on the same inputs on the same GPU as this build's kernels.

Known reference behaviour excluded here (and documented): with --use_fast_math the reference's fused
GEMM flushes s_inv = 2^-127 to zero for rows whose max is zero or below 2^-113, then multiplies by
1/0 and returns NaN for those rows; this build keeps the exact subnormal and returns the bias."""
import math
import pathlib

import pytest
import torch
import torch.nn.functional as F

import inputs
from helpers import (assert_close_ulp, bf16_ulp, bits_equal, edge_rows, gemm_tolerance, rel_err, report,
                     ulp_distance)

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
    # within one bf16 ulp of the reference's output wherever the two fp32 accumulations (different
    # orders) cannot move the value by half an ulp; elsewhere the tolerance above applies
    dist = ulp_distance(y, y_ref)
    acc_bound = 2 * 8.0 * math.sqrt(K) * 2.0 ** -24 * absprod.cpu()
    tight = acc_bound < 0.5 * bf16_ulp(y_ref.cpu())
    assert int(dist[tight].max()) <= 1, f"{int((dist[tight] > 1).sum())} well-conditioned elements beyond 1 ulp"
    exact = x.double() @ w.double().t() + b.double()
    report(f"linear vs reference fused kernel {M}x{K}x{N}", bit_equal=float((dist == 0).double().mean()),
           within_1ulp=float((dist <= 1).double().mean()), max_ulp=int(dist.max()),
           max_ulp_well_conditioned=int(dist[tight].max()), well_conditioned=float(tight.double().mean()),
           err_fp64=rel_err(y, exact), ref_err_fp64=rel_err(y_ref, exact))
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


def _reference_sdpa(small, q, k, v, causal):
    """The reference's inference attention (tbf16/attention.py:38-65) on the GPU: its own head_amax and
    head_scale_cast kernels for the exponents and the fp16 copies (v_exp = 13), torch's fp16 attention on
    the memory-efficient backend, and its head_scale_cast of the fp16 output back to bf16."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    B, H = q.shape[:2]
    Hkv = k.shape[1]
    eq = torch.frexp(small.head_amax(q))[1].amax()
    ek = torch.frexp(small.head_amax(k))[1].amax()
    a = torch.div(ek - eq, 2, rounding_mode="floor")
    a = torch.maximum(torch.minimum(a, 14 - eq), ek - 14).to(torch.int32)
    ev = (torch.frexp(small.head_amax(v))[1] - 13).to(torch.int32)
    q16 = small.head_scale_cast(q, a.expand(B, H).contiguous(), torch.float16)
    k16 = small.head_scale_cast(k, (-a).expand(B, Hkv).contiguous(), torch.float16)
    v16 = small.head_scale_cast(v, (-ev).contiguous(), torch.float16)
    with sdpa_kernel(SDPBackend.EFFICIENT_ATTENTION):
        out16 = F.scaled_dot_product_attention(q16, k16, v16, is_causal=causal, enable_gqa=H != Hkv)
    ev_q = ev if H == Hkv else ev.repeat_interleave(H // Hkv, 1)
    return small.head_scale_cast(out16, ev_q.contiguous(), torch.bfloat16), q16, k16, v16, ev_q


def _attention_tolerance(q16, k16, v16, ev_q, out_ref, causal, rows_per_chunk=2048):
    """Per-element bound between two fp16 attention pipelines, computed on the GPU in fp64: one bf16 ulp,
    the fp16 rounding of P in each (2^-10 of the head's V scale), and the fp32 rounding of the logits in
    each (4 ulp of the row's largest |logit| times the weights' spread, which matters for config 3's
    logits that overflow fp16)."""
    B, H, S, D = q16.shape
    grp = H // k16.shape[1]
    scale = 1.0 / math.sqrt(D)
    two_ev = torch.ldexp(torch.ones((), device=q16.device, dtype=torch.float64), ev_q.double())
    tol = torch.empty(out_ref.shape, dtype=torch.float64, device=q16.device)
    for b in range(B):
        for h in range(H):
            kh, vh = k16[b, h // grp].double(), v16[b, h // grp].double()
            vmax = vh.abs().amax()
            for r0 in range(0, S, rows_per_chunk):
                r1 = min(S, r0 + rows_per_chunk)
                s = (q16[b, h, r0:r1].double() @ kh.t()) * scale
                if causal:
                    s.masked_fill_(torch.arange(S, device=s.device)[None, :] > torch.arange(r0, r1, device=s.device)[:, None],
                                   float("-inf"))
                zmax = torch.where(torch.isfinite(s), s.abs(), torch.zeros_like(s)).amax(-1, keepdim=True)
                p = torch.softmax(s, -1)
                spread = p @ vh.abs() + (p @ vh).abs()
                tol[b, h, r0:r1] = (2.0 ** -10 * vmax + 2.0 ** -20 * zmax * spread) * two_ev[b, h]
    return tol + bf16_ulp(out_ref).to(tol.device)


@pytest.mark.parametrize("S", [4096, 16384])
@pytest.mark.parametrize("causal", [False, True])
def test_sdpa_vs_reference_pipeline_config3(S, causal):
    """Config 3 (B=1, H=16, D=128, Q/K x 2^8 so raw logits overflow fp16, V x 2^h per head) at full size:
    every output element against the reference's own pipeline run on the same GPU."""
    from tbf16 import attention
    small = _ref("tbf16_ref_small")
    q, k, v = inputs.attention_qkv(1, 16, S, 128, seed=S + int(causal), device="cuda")
    out = attention.sdpa(q, k, v, is_causal=causal)
    out_ref, q16, k16, v16, ev_q = _reference_sdpa(small, q, k, v, causal)
    q16m, k16m, v16m, _, _ = attention.prepare_qkv(q, k, v, v_exp=13)
    assert bits_equal(q16m, q16) and bits_equal(k16m, k16) and bits_equal(v16m, v16)
    tol = _attention_tolerance(q16, k16, v16, ev_q, out_ref, causal)
    d = (out.double() - out_ref.double()).abs()
    dist = ulp_distance(out, out_ref)
    report(f"sdpa vs reference pipeline S={S} causal={causal}", bit_equal=float((dist == 0).double().mean()),
           within_1ulp=float((dist <= 1).double().mean()), max_ulp=int(dist.max()),
           worst_over_tol=float((d / tol).max()))
    assert torch.isfinite(out.float()).all()
    assert (d <= tol).all(), f"{int((d > tol).sum())} elements outside tolerance"
    assert float((dist <= 1).double().mean()) > 0.99
