"""Training path parity: tbf16.autograd.linear (ScaledLinearFn) and tbf16.autograd.sdpa (ScaledSDPAFn)
against the oracle's fp64 restatement of the reference's algorithm (autograd.py:58-90, 149-193) on the
same seeded inputs (elementwise), and against plain fp64 autograd (relative error below 2e-3). Cases
follow the reference's tests/test_autograd.py: gaussian, tiny and huge gradients, odd sizes, long M,
GQA, causal, dO x1e-10, dO x1e6 with v x1e4, peaky q/k, and boolean / float sliding-window + padding
masks, at head dims 64, 128 and 256 (and 200, zero-padded)."""
import math

import pytest
import torch
import torch.nn.functional as F

from helpers import assert_close_ulp, bf16_ulp, gemm_tolerance, rel_err, report
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _grads(fn, inputs, dout):
    ins = [t.detach().clone().requires_grad_() for t in inputs]
    out = fn(*ins)
    out.backward(dout)
    return [out] + [t.grad for t in ins]


@pytest.mark.parametrize("name,M,K,N,xs,gs", [("gaussian", 2048, 1024, 768, 1.0, 1.0),
                                              ("grads x1e-12", 2048, 1024, 768, 1.0, 1e-12),
                                              ("grads x1e8, x x1e4", 2048, 1024, 768, 1e4, 1e8),
                                              ("M=33 K=520 N=72", 33, 520, 72, 1.0, 1.0),
                                              ("long M", 40000, 256, 256, 1.0, 1.0)])
def test_linear_train(name, M, K, N, xs, gs):
    from tbf16 import autograd as ag
    g = torch.Generator().manual_seed(M + K + N)
    x = (torch.randn(M, K, generator=g) * xs).bfloat16()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).bfloat16()
    b = torch.randn(N, generator=g).bfloat16()
    dy = (torch.randn(M, N, generator=g) * gs).bfloat16()
    y, dx, dw, db = _grads(ag.linear, [x.cuda(), w.cuda(), b.cuda()], dy.cuda())
    ref = orc.linear_train(x, w, b, dy)
    # elementwise against the oracle (same exponents, fp64 accumulation)
    assert_close_ulp(y.cpu(), ref["y"], gemm_tolerance(ref["y"], x.double().abs() @ w.double().abs().t(), K), what="y")
    assert_close_ulp(dx.cpu(), ref["dx"], gemm_tolerance(ref["dx"], dy.double().abs() @ w.double().abs(), N), what="dx")
    assert_close_ulp(dw.cpu(), ref["dw"], gemm_tolerance(ref["dw"], dy.double().abs().t() @ x.double().abs(), M),
                     what="dw")
    # and against plain fp64 autograd
    e_y, e_dx, e_dw, e_db = _grads(F.linear, [x.double(), w.double(), b.double()], dy.double())
    errs = {}
    for got, exact, what in ((y, e_y, "y"), (dx, e_dx, "dx"), (dw, e_dw, "dw"), (db, e_db, "db")):
        assert torch.isfinite(got.float()).all(), what
        errs[what] = rel_err(got, exact)
    report(f"linear_train {name} vs fp64", **errs)
    for what, e in errs.items():
        assert e < 2e-3, (what, e)


def _ref_attn(q, k, v, causal, allowed=None):
    H = q.shape[1]
    if k.shape[1] != H:
        k = k.repeat_interleave(H // k.shape[1], 1)
        v = v.repeat_interleave(H // v.shape[1], 1)
    s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    if causal:
        S = s.shape[-1]
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    if allowed is not None:
        s = s.masked_fill(~allowed, float("-inf"))
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize("name,Hq,Hkv,S,D,causal,qs,gs,vs", [
    ("gaussian", 8, 8, 1024, 64, False, 1.0, 1.0, 1.0),
    ("causal", 8, 8, 1024, 128, True, 1.0, 1.0, 1.0),
    ("GQA 16/4 causal", 16, 4, 1024, 128, True, 1.0, 1.0, 1.0),
    ("dO x1e-10", 8, 8, 1024, 64, True, 1.0, 1e-10, 1.0),
    ("dO x1e6, v x1e4", 8, 8, 1024, 64, True, 1.0, 1e6, 1e4),
    ("peaky q,k x8", 8, 8, 1024, 64, True, 8.0, 1.0, 1.0),
    ("odd length", 4, 2, 333, 64, True, 1.0, 1.0, 1.0),
    ("D=256 GQA 8/4 causal", 8, 4, 1024, 256, True, 1.0, 1.0, 1.0),
    ("D=256 non-causal", 4, 4, 512, 256, False, 1.0, 1.0, 1.0),
    ("D=256 dO x1e-10, v x1e4", 4, 2, 512, 256, True, 1.0, 1e-10, 1e4),
    ("D=256 odd length", 4, 2, 333, 256, True, 1.0, 1.0, 1.0),
    ("D=200 padded to 256", 2, 2, 256, 200, True, 1.0, 1.0, 1.0)])
def test_sdpa_train(name, Hq, Hkv, S, D, causal, qs, gs, vs):
    from tbf16 import autograd as ag
    g = torch.Generator().manual_seed(Hq * S + D)
    q = (torch.randn(1, Hq, S, D, generator=g) * qs).bfloat16()
    k = (torch.randn(1, Hkv, S, D, generator=g) * qs).bfloat16()
    v = (torch.randn(1, Hkv, S, D, generator=g) * vs).bfloat16()
    do = (torch.randn(1, Hq, S, D, generator=g) * gs).bfloat16()
    gqa = Hq != Hkv
    o, dq, dk, dv = _grads(lambda q, k, v: ag.sdpa(q, k, v, is_causal=causal, enable_gqa=gqa),
                           [q.cuda(), k.cuda(), v.cuda()], do.cuda())
    ref = orc.sdpa_bwd(q, k, v, do, is_causal=causal)
    exact = _grads(lambda q, k, v: _ref_attn(q, k, v, causal), [q.double(), k.double(), v.double()], do.double())
    # elementwise against the oracle: one bf16 ulp plus the fp16 rounding of P (2^-10 of the head's V scale)
    # for the output, and for the gradients 2^-9 of the magnitudes the fp16 rounding of P, delta and dS
    # scale with (oracle abs_dq / abs_dk / abs_dv), plus 2^-24 of what fp16's rounding near zero scales
    # with (sub_dq / sub_dk / sub_dv: P or dS below fp16's smallest subnormal flush to zero)
    f = orc.sdpa_fwd(q, k, v, is_causal=causal, v_exp=0)
    vmax = orc._expand_kv(v.double().abs().amax(dim=(-2, -1), keepdim=True), Hq)
    two_ev = torch.ldexp(torch.ones(()), orc.expand_heads(f["ev"], Hq).double())[..., None, None]
    tols = {"o": bf16_ulp(ref["out"]) + 2.0 ** -10 * vmax
                 + 2.0 ** -21 * f["zmax"][..., None] * (f["pv_abs"] + f["o16"].abs()) * two_ev,
            "dq": bf16_ulp(ref["dq"]) + 2.0 ** -9 * ref["abs_dq"] + 2.0 ** -24 * ref["sub_dq"],
            "dk": bf16_ulp(ref["dk"]) + 2.0 ** -9 * ref["abs_dk"] + 2.0 ** -24 * ref["sub_dk"],
            "dv": bf16_ulp(ref["dv"]) + 2.0 ** -9 * ref["abs_dv"] + 2.0 ** -24 * ref["sub_dv"]}
    errs, worst = {}, {}
    for got, orc_v, ex, what in ((o, ref["out"], exact[0], "o"), (dq, ref["dq"], exact[1], "dq"),
                                 (dk, ref["dk"], exact[2], "dk"), (dv, ref["dv"], exact[3], "dv")):
        assert torch.isfinite(got.float()).all(), what
        errs[what] = rel_err(got, ex)
        d = (got.cpu().double() - orc_v.double()).abs()
        worst[what] = float((d / tols[what]).max())
    report(f"sdpa_train {name} vs fp64", **errs)
    report(f"sdpa_train {name} vs oracle, worst error / tolerance", **worst)
    for what in errs:
        assert worst[what] <= 1.0, (what, worst[what])
        assert errs[what] < 2e-3, (what, errs[what])


def test_sdpa_train_exponent_G_bit_exact():
    """The per-call dO exponent G (autograd.py:175-178) is computed on the device and matches the oracle."""
    from tbf16 import attention, autograd as ag
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(2, 4, 256, 64, generator=g).bfloat16() for _ in range(3))
    for gs in (1.0, 1e-10, 3e5):
        do = (torch.randn(2, 4, 256, 64, generator=g) * gs).bfloat16()
        q16, k16, v16, a, ev = attention.prepare_qkv(q.cuda(), k.cuda(), v.cuda())
        out, lse, o16 = attention.attn_forward(q16, k16, v16, ev, need_lse=True, need_o16=True)
        *_, G = ag.attn_backward(q16, k16, v16, o16, lse, a, ev, do.cuda(), None, False, 1 / 8, 64)
        assert int(G) == orc.sdpa_bwd(q, k, v, do)["G"]


@pytest.mark.parametrize("kind,D", [("bool", 64), ("float", 64), ("bool", 256)])
def test_sdpa_train_masks(kind, D):
    """Sliding window + padding (reference tests/test_autograd.py:45-64)."""
    from tbf16 import autograd as ag
    Hq, Hkv, S = 8, 4, 1000
    g = torch.Generator().manual_seed(7)
    q = torch.randn(2, Hq, S, D, generator=g).bfloat16()
    k, v = (torch.randn(2, Hkv, S, D, generator=g).bfloat16() for _ in range(2))
    do = torch.randn(2, Hq, S, D, generator=g).bfloat16()
    i = torch.arange(S)
    allowed = (i[None, :] <= i[:, None]) & (i[:, None] - i[None, :] < 256)
    allowed = allowed[None, None].expand(2, 1, S, S).clone()
    allowed[1, :, :, 700:] = False
    allowed[1, :, :, 0] = True
    mask = allowed if kind == "bool" else torch.zeros(allowed.shape).masked_fill(~allowed, float("-inf")).bfloat16()
    o, dq, dk, dv = _grads(lambda q, k, v: ag.sdpa(q, k, v, attn_mask=mask.cuda(), enable_gqa=True),
                           [q.cuda(), k.cuda(), v.cuda()], do.cuda())
    exact = _grads(lambda q, k, v: _ref_attn(q, k, v, False, allowed), [q.double(), k.double(), v.double()], do.double())
    errs = {}
    for got, ex, what in zip((o, dq, dk, dv), exact, ("o", "dq", "dk", "dv")):
        assert torch.isfinite(got.float()).all(), what
        errs[what] = rel_err(got, ex)
    report(f"sdpa_train masks {kind} D={D} vs fp64", **errs)
    for what, e in errs.items():
        assert e < 2e-3, (what, e)
