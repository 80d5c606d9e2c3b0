"""Training parity on config 4's own shapes: the SwiGLU MLP's linears (M = 8192 tokens, hidden 2048,
intermediate 8192) and causal attention (B = 2, 16 heads of D = 128, S = 4096), with the upstream
gradient dY = N(0, 1) * 2^-20 that exercises the power-of-two scaling of dY and dO.

Each gradient is checked three ways:
  * against fp64 at full size (computed on the GPU in float64): relative error below 2e-3, the bound
    the training path is held to;
  * elementwise against the oracle (the reference's algorithm, tbf16/autograd.py:58-90 and :149-193,
    restated in fp64 on the exact fp16 operands) on sampled output rows / heads, with every scale
    exponent taken over the full tensors;
  * for attention, against the reference's own GPU pipeline on the same inputs: its fp16 operands
    (bit-equal to this build's), torch's fp16 memory-efficient attention forward / backward with the
    dO exponent G and the fp16 dq16 / dk16 / dv16 it produces (autograd.py:153-193); this build must be
    at least as close to fp64 as that pipeline.
"""
import math

import pytest
import torch

from helpers import assert_close_ulp, bf16_ulp, gemm_tolerance, rel_err, report
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL_FP64 = 2e-3
M_TOKENS, HIDDEN, INTER = 8192, 2048, 8192


def _grads(fn, inputs, dout):
    ins = [t.detach().clone().requires_grad_() for t in inputs]
    out = fn(*ins)
    out.backward(dout)
    return [out.detach()] + [t.grad for t in ins]


@pytest.mark.parametrize("layer,K,N", [("gate/up", HIDDEN, INTER), ("down", INTER, HIDDEN)])
def test_config4_mlp_linear(layer, K, N):
    from tbf16 import autograd as ag
    M = M_TOKENS
    g = torch.Generator().manual_seed(400 + K)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    dy = (torch.randn(M, N, generator=g) * 2.0 ** -20).bfloat16()
    xc, wc, dyc = x.cuda(), w.cuda(), dy.cuda()
    y, dx, dw = _grads(lambda a, b: ag.linear(a, b), [xc, wc], dyc)
    for t, what in ((y, "y"), (dx, "dx"), (dw, "dw")):
        assert torch.isfinite(t.float()).all(), what

    # fp64 at full size, on the GPU
    xd, wd, dyd = xc.double(), wc.double(), dyc.double()
    errs = {"y": rel_err(y, xd @ wd.t()), "dx": rel_err(dx, dyd @ wd), "dw": rel_err(dw, dyd.t() @ xd)}
    del xd, wd, dyd

    # elementwise against the oracle on 128 sampled rows of y / dx and 128 sampled rows of dw
    rows = torch.randperm(M, generator=g)[:128].sort().values
    dw_rows = torch.randperm(N, generator=g)[:128].sort().values
    ref = orc.linear_train(x, w, None, dy, rows=rows, dw_rows=dw_rows)
    xa, wa, dya = x.double().abs(), w.double().abs(), dy.double().abs()
    checks = ((y.cpu()[rows], ref["y"], xa[rows] @ wa.t(), K, "y"),
              (dx.cpu()[rows], ref["dx"], dya[rows] @ wa, N, "dx"),
              (dw.cpu()[dw_rows], ref["dw"], dya[:, dw_rows].t() @ xa, M, "dw"))
    for got, want, absprod, kk, what in checks:
        assert_close_ulp(got, want, gemm_tolerance(want, absprod, kk), frac_exact=0.9, what=f"{layer} {what}")
    report(f"config4 linear {layer} vs fp64", **errs)
    for what, e in errs.items():
        assert e < TOL_FP64, (layer, what, e)


def _attention_fp64(q, k, v, do, causal, scale):
    """Exact attention forward / backward in float64 on the GPU, one head at a time."""
    B, H, S, D = q.shape
    grp = H // k.shape[1]
    o, dq = torch.empty_like(q, dtype=torch.float64), torch.empty_like(q, dtype=torch.float64)
    dk, dv = torch.zeros_like(k, dtype=torch.float64), torch.zeros_like(v, dtype=torch.float64)
    keep = torch.ones(S, S, dtype=torch.bool, device=q.device).tril() if causal else None
    for b in range(B):
        for h in range(H):
            qh, kh, vh, doh = q[b, h].double(), k[b, h // grp].double(), v[b, h // grp].double(), do[b, h].double()
            s = (qh @ kh.t()) * scale
            if keep is not None:
                s.masked_fill_(~keep, float("-inf"))
            p = torch.softmax(s, -1)
            oh = p @ vh
            dp = doh @ vh.t()
            ds = p * (dp - (doh * oh).sum(-1, keepdim=True))
            o[b, h] = oh
            dq[b, h] = (ds @ kh) * scale
            dk[b, h // grp] += (ds.t() @ qh) * scale
            dv[b, h // grp] += p.t() @ doh
    return o, dq, dk, dv


def _reference_pipeline(q, k, v, do, causal, scale):
    """The reference's training attention (tbf16/autograd.py:149-193) on the GPU: fp16 operands from
    prepare_qkv (this build's tbf16_prepare_qkv, bit-equal to the reference's, see
    test_gpu_reference_kernels.py), torch's fp16 memory-efficient attention forward and backward, the
    global dO exponent G, and the fp16 dq16 / dk16 / dv16 scaled back to bf16 (head_scale)."""
    from tbf16 import attention
    H, Hkv, D = q.shape[1], k.shape[1], q.shape[-1]
    q16, k16, v16, a, ev = attention.prepare_qkv(q, k, v)
    rep = lambda t: t if t.shape[1] == H else t.repeat_interleave(H // t.shape[1], 1)
    out16, lse, seed, off = torch.ops.aten._scaled_dot_product_efficient_attention(
        q16, rep(k16), rep(v16), None, True, 0.0, causal, scale=scale)
    ev_q = attention.expand_heads(ev, H)
    G = (12 - math.ceil(math.log2(D))) - (attention.head_exp(do) + ev_q).amax()
    do16 = attention.head_scale(do, ev_q + G, torch.float16)
    dq16, dk16, dv16, _ = torch.ops.aten._scaled_dot_product_efficient_attention_backward(
        do16, q16, rep(k16), rep(v16), None, out16, lse, seed, off, 0.0, [True, True, True, False], causal,
        scale=scale)
    red = lambda t: t if H == Hkv else t.float().view(t.shape[0], Hkv, H // Hkv, *t.shape[2:]).sum(2)
    assert torch.isfinite(dq16).all() and torch.isfinite(dk16).all() and torch.isfinite(dv16).all()
    return (attention.head_scale(out16, ev_q, torch.bfloat16), attention.head_scale(dq16, a - G, torch.bfloat16),
            attention.head_scale(red(dk16), -a - G, torch.bfloat16),
            attention.head_scale(red(dv16), -ev - G, torch.bfloat16))


def test_config4_attention():
    from tbf16 import autograd as ag
    B, H, S, D = 2, 16, 4096, 128
    causal, scale = True, 1.0 / math.sqrt(D)
    g = torch.Generator().manual_seed(4004)
    q, k, v = (torch.randn(B, H, S, D, generator=g).bfloat16() for _ in range(3))
    do = (torch.randn(B, H, S, D, generator=g) * 2.0 ** -20).bfloat16()
    qc, kc, vc, doc = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    got = _grads(lambda a, b, c: ag.sdpa(a, b, c, is_causal=causal), [qc, kc, vc], doc)
    names = ("o", "dq", "dk", "dv")
    for t, what in zip(got, names):
        assert torch.isfinite(t.float()).all(), what

    exact = _attention_fp64(qc, kc, vc, doc, causal, scale)
    errs = {n: rel_err(t, e) for n, t, e in zip(names, got, exact)}
    ref_errs = {}
    try:
        refp = _reference_pipeline(qc, kc, vc, doc, causal, scale)
        ref_errs = {n: rel_err(t, e) for n, t, e in zip(names, refp, exact)}
    except RuntimeError as exc:  # torch built without a memory-efficient kernel for this GPU
        report("config4 attention reference pipeline unavailable", reason=str(exc).splitlines()[0][:80])
    del exact

    # elementwise against the oracle on two (batch, head) pairs; exponents over all heads
    heads = [(0, 3), (1, 12)]
    ref = orc.sdpa_bwd(q, k, v, do, is_causal=causal, kv_heads=heads)
    pick = lambda t: torch.stack([t[b, h:h + 1].cpu() for b, h in heads])
    # gradients: one bf16 ulp plus 2^-9 of the magnitudes the fp16 rounding of P, delta (from fp16 O) and
    # dS scale with, plus 2^-24 of what fp16's absolute rounding near zero scales with
    # forward: one ulp, the fp16 rounding of P (2^-10 of the head's V scale) and the fp32 logits' rounding
    vmax = torch.stack([v[b, h:h + 1] for b, h in heads]).double().abs().amax(dim=(-2, -1), keepdim=True)
    two_ev = torch.ldexp(torch.ones(()), ref["ev"].double())[..., None, None]
    f = orc.sdpa_fwd(q, k, v, is_causal=causal, v_exp=0, kv_heads=heads)
    tol_o = (bf16_ulp(ref["out"]) + 2.0 ** -10 * vmax
             + 2.0 ** -21 * f["zmax"][..., None] * (f["pv_abs"] + f["o16"].abs()) * two_ev)
    del f
    worst = {}
    grad_tol = lambda n: bf16_ulp(ref[n]) + 2.0 ** -9 * ref["abs_" + n] + 2.0 ** -24 * ref["sub_" + n]
    for what, t, want, tol in (("o", got[0], ref["out"], tol_o), ("dq", got[1], ref["dq"], grad_tol("dq")),
                               ("dk", got[2], ref["dk"], grad_tol("dk")), ("dv", got[3], ref["dv"], grad_tol("dv"))):
        d = (pick(t).double() - want.double()).abs()
        worst[what] = float((d / tol).max())
        assert (d <= tol).all(), f"{what}: {int((d > tol).sum())} elements outside tolerance, worst {worst[what]:.2f}x"
    report("config4 attention vs fp64", **errs)
    if ref_errs:
        report("config4 attention reference pipeline vs fp64", **ref_errs)
    report("config4 attention vs oracle, worst error / tolerance", **worst)
    for n in names:
        assert errs[n] < TOL_FP64, (n, errs[n])
        if ref_errs:
            assert errs[n] <= ref_errs[n] * 1.02, (n, errs[n], ref_errs[n])
