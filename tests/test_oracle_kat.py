"""Known-answer tests for the oracle's exponent and rounding rules, derived from the reference's
CUDA lines (the reference ships no such tests): tbf16/csrc/small_kernels.cu:12-18,
tbf16/csrc/gemm_sm75.cu:19-23, tbf16/ops.py:29-32, torch.frexp as used by attention.py:27."""
import math
import struct

import pytest
import torch


def bits(f):
    return struct.unpack("<I", struct.pack("<f", f))[0]


def fl(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


SUB = fl(0x00000100)  # an fp32 subnormal


@pytest.mark.parametrize("amax,t,expect_log2", [
    (0.0, 0, 125),            # e clamps to 1 -> se = 252
    (0.0, 15, 127),           # se = 267 clamps to 254
    (SUB, 0, 125),            # subnormal amax behaves like zero
    (1.0, 0, -1),             # 1.0 * 2^-1 = 0.5 in [0.5, 1)
    (0.99999, 0, 0),
    (0.5, 0, 0),
    (65504.0, 0, -16),
    (1.0, 15, 14),            # L1/max target 2^15
    (float("inf"), 0, -126),  # e = 255 clamps to 252 -> se = 1
    (float("nan"), 0, -126),
    (3.0e38, 15, -111),       # e = 254 -> clamps to 252 -> se = 16
    (1.0, -1, -2),
])
def test_pow2_scale_small(orc, amax, t, expect_log2):
    s = orc.pow2_scale(torch.tensor([amax]), t, "small")[0].item()
    assert s == 2.0 ** expect_log2


@pytest.mark.parametrize("amax,expect_log2", [
    (0.0, 127),               # min(253 + 15 - 1, 254) = 254
    (1.0, 14),                # 1 * 2^14 in [2^14, 2^15)
    (65504.0, -1),            # 32752
    (2.0 ** -100, 114),
    (float("inf"), -111),     # e clamps to 252 -> 16
    (1e-40, 127),
])
def test_pow2_scale_fused(orc, amax, expect_log2):
    s = orc.pow2_scale(torch.tensor([amax]), 15, "fused")[0].item()
    assert s == 2.0 ** expect_log2


def test_pow2_scale_bins(orc):
    """Every normal amax lands in [2^(t-1), 2^t) after scaling, at and around bin edges."""
    vals = []
    for e in range(-120, 120):
        for m in (1.0, 1.0 + 2 ** -23, 2.0 - 2 ** -23):
            vals.append(m * 2.0 ** e)
    a = torch.tensor(vals, dtype=torch.float32)
    for t in (0, -1, -3, 15):
        s = orc.pow2_scale(a, t, "small")
        y = a.double() * s.double()
        ok = (y >= 2.0 ** (t - 1)) & (y < 2.0 ** t)
        eb = torch.floor(torch.log2(a.double())) + 127
        unclamped = (253 + t - eb >= 1) & (253 + t - eb <= 254)   # scale exponent inside [1, 254]
        assert ok[unclamped].all() and unclamped.sum() > 200
        sf = orc.pow2_scale(a, 15, "fused")
        yf = a.double() * sf.double()
        assert ((yf >= 2.0 ** 14) & (yf < 2.0 ** 15))[a >= 2.0 ** -113].all()  # below: scale clamps at 2^127


def test_triton_formula_matches_small_for_normal_amax(orc):
    a = torch.exp2(torch.arange(-100, 100, dtype=torch.float32)) * 1.37
    for t in (0, -1, 15):
        assert torch.equal(orc.pow2_scale(a, t, "small"), orc.pow2_scale(a, t, "triton"))


@pytest.mark.parametrize("x,e", [(0.0, 0), (1.0, 1), (0.5, 0), (3.0, 2), (0.75, 0), (2.0 ** -140, -139),
                                 (float("inf"), 0), (float("nan"), 0), (65504.0, 16), (-4.0, 3)])
def test_frexp_exp(orc, x, e):
    assert orc.frexp_exp(torch.tensor([x]))[0].item() == e
    if math.isfinite(x):
        assert torch.frexp(torch.tensor([x]))[1].item() == e


def test_f16_rounding_edges(orc):
    cases = {65504.0: 0x7BFF, 65519.0: 0x7BFF, 65520.0: 0x7C00, 2.0 ** -24: 0x0001, 2.0 ** -25: 0x0000,
             1.5 * 2.0 ** -25: 0x0001, 2.0 ** -14: 0x0400, 1.0 + 2 ** -11: 0x3C00, 1.0 + 3 * 2 ** -11: 0x3C02,
             -0.0: 0x8000, float("inf"): 0x7C00}
    x = torch.tensor(list(cases.keys()), dtype=torch.float32)
    got = orc.f16_rn(x).view(torch.int16).numpy().astype("uint16").tolist()
    assert got == list(cases.values())


def test_f16_rounding_matches_torch(orc):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(200000, generator=g) * torch.exp2(torch.randint(-40, 20, (200000,), generator=g).float())
    assert torch.equal(orc.f16_rn(x).view(torch.int16), x.half().view(torch.int16))
    assert torch.equal(orc.bf16_rn(x).view(torch.int16), x.bfloat16().view(torch.int16))


def test_target_exp(orc, golden):
    for K, t in zip(golden["target_exp_K"], golden["target_exp_t"]):
        assert orc.target_exp(int(K)) == int(t)


def test_row_reduce_l1_exact(orc):
    """The L1 norm is the exact sum rounded once: 2^24 ones and a 1 that fp32 summation would drop."""
    x = torch.tensor([[1.0] + [2.0 ** -24] * 4 + [0.0] * 3], dtype=torch.bfloat16)
    assert orc.row_reduce(x, l1=True)[0].item() == 1.0 + 2 ** -22
    y = torch.tensor([[float("nan"), 2.0, -3.0, 1.0]], dtype=torch.bfloat16)
    assert orc.row_reduce(y, l1=False)[0].item() == 3.0  # fmaxf ignores NaN


def test_fused_rows_oracle_known_answers():
    from oracle import oracle as orc
    """The producer-fusion restatements on hand-checked rows: silu(0) = 0 and silu(g) * 1 = bf16(silu(g));
    a constant row's RMSNorm is 1 (times weight + 1 = 1), whose row max 1 gets the fused rule's scale
    2^14 at t = 15 (biased exponent 253 + 15 - 127 = 141)."""
    g = torch.tensor([[0.0, 1.0, -1.0, 2.0, 0.5, -0.5, 4.0, -4.0]]).bfloat16()
    u = torch.ones_like(g)
    h16, s_inv, h = orc.glu_rows(g, u, "silu")
    assert h[0, 0].item() == 0.0
    ref = (g.float() / (1 + torch.exp(-g.float()))).bfloat16()
    assert torch.equal(h, ref)
    x = torch.full((1, 8), 3.0).bfloat16()
    w = torch.zeros(8).bfloat16()
    r16, s_inv, r = orc.rmsnorm_rows(x, w, eps=0.0, offset=1.0, style="gemma")
    assert torch.all(r.float() == 1.0)  # x / rms(x) = 1, times (0 + 1)
    assert s_inv.item() == 2.0 ** -14  # row max 1 -> biased 127 -> scale 2^(253 + 15 - 127 - 127)
    assert torch.all(r16.float() == 2.0 ** 14)


def test_fused_op_restatements_match_torch_cpu():
    """The oracle's restatements of the fused model-side ops against torch's own bf16 ops on the CPU:
    rotary embedding and the residual add bit-equal; the gated activation's backward within one bf16
    ulp of torch's autograd (its CPU exp / tanh may differ from the oracle's in the last fp32 bit)."""
    import torch.nn.functional as F
    from oracle import oracle as orc
    g = torch.Generator().manual_seed(3)
    S, H, D = 9, 2, 64
    y = (torch.randn(2, S, H, D, generator=g) * 3).bfloat16()
    ang = torch.outer(torch.arange(S, dtype=torch.float32), 1.0 / (1e4 ** (torch.arange(0, D, 2) / D)))
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16()
    rot = torch.cat([-y[..., D // 2:], y[..., :D // 2]], -1)
    ref = y * cos[:, None, :] + rot * sin[:, None, :]
    assert torch.equal(orc.rope(y, cos, sin).view(torch.int16), ref.view(torch.int16))
    x = torch.randn(5, 64, generator=g).bfloat16()
    res = (torch.randn(5, 64, generator=g) * 10).bfloat16()
    w = (torch.randn(64, generator=g) * 0.1).bfloat16()
    s, r16, s_inv = orc.add_rmsnorm_rows(x, res, w)
    assert torch.equal(s.view(torch.int16), (res + x).view(torch.int16))
    r16b, s_invb, _ = orc.rmsnorm_rows(res + x, w)
    assert torch.equal(r16.view(torch.int16), r16b.view(torch.int16)) and torch.equal(s_inv, s_invb)
    for act in ("silu", "gelu_tanh"):
        gt = (torch.randn(7, 256, generator=g) * 3).bfloat16().requires_grad_()
        ut = torch.randn(7, 256, generator=g).bfloat16().requires_grad_()
        dh = (torch.randn(7, 256, generator=g) * 0.01).bfloat16()
        h = (F.silu(gt) if act == "silu" else F.gelu(gt, approximate="tanh")) * ut
        h.backward(dh)
        dg, du = orc.glu_bwd(dh, gt.detach(), ut.detach(), act)
        # where tanh saturates (g < -5) torch's CPU kernel rounds tanh to exactly -1, giving 0 where the
        # restatement keeps a value below 1e-7: an absolute floor of 2^-18 max|dh| covers that
        floor = 2.0 ** -18 * dh.abs().max().item()
        for ours, theirs in ((dg, gt.grad), (du, ut.grad)):
            d = (ours.double() - theirs.double()).abs()
            assert bool((d <= orc.bf16_ulp(theirs.double()) + floor).all()), act
