"""Producer fusion (glu_rows / rmsnorm_rows and the linears they feed): the kernel's bf16 rows within one
bf16 ulp of the oracle's fp32 restatement (the activation / rsqrt functions of the GPU and of the host
may differ in the last fp32 bit), its row scales and fp16 operands bit-exact for the rows it produced
(the fused rule, as tbf16_row_scale), and glu_linear / rmsnorm_linear bit-equal to scaled_linear on
those rows. Called through tbf16.ops (ctypes -> C ABI)."""
import pytest
import torch

from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _within_ulp(a, b):
    d = (a.double() - b.double()).abs()
    return bool((d <= orc.bf16_ulp(b.double())).all())


def _gate_up(M, I, seed):
    g = torch.Generator().manual_seed(seed)
    gate = (torch.randn(M, I, generator=g) * 3).bfloat16()
    up = (torch.randn(M, I, generator=g) * torch.exp2(torch.randint(-8, 8, (M, 1), generator=g).float())).bfloat16()
    return gate, up


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
# one warp per row up to 1024 elements (1, 2 or 4 vectors a lane; row counts not a multiple of the 8 rows
# of a block), one right-sized block per row above (one or two vectors a thread)
@pytest.mark.parametrize("M,I", [(1, 8), (9, 384), (13, 1000), (5, 2056), (64, 8192), (3, 10240), (17, 16384)])
def test_glu_rows(act, M, I):
    from tbf16 import ops
    gate, up = _gate_up(M, I, M + I)
    h16, s_inv, h = ops.glu_rows(gate.cuda(), up.cuda(), act, want_h=True)
    h16, s_inv, h = h16.cpu(), s_inv.cpu(), h.cpu()
    _, _, h_ref = orc.glu_rows(gate, up, act)
    assert _within_ulp(h, h_ref)
    assert (h.view(torch.int16) == h_ref.view(torch.int16)).float().mean() > 0.999
    assert torch.equal(s_inv, orc.row_scale_fused(h, 15))  # the fused rule on the produced rows
    assert torch.equal(h16.view(torch.int16), orc.f16_rn(h.float() / s_inv[:, None]).view(torch.int16))


def test_glu_rows_match_torch_on_gpu():
    """The fused rows against torch's own act(g) * u on the GPU (bf16 tensors)."""
    import torch.nn.functional as F
    from tbf16 import ops
    gate, up = _gate_up(128, 4096, 7)
    g, u = gate.cuda(), up.cuda()
    for act, ref in (("silu", F.silu(g) * u), ("gelu_tanh", F.gelu(g, approximate="tanh") * u)):
        _, _, h = ops.glu_rows(g, u, act, want_h=True)
        assert _within_ulp(h.cpu(), ref.cpu())
        assert (h.view(torch.int16) == ref.view(torch.int16)).float().mean().item() > 0.999


@pytest.mark.parametrize("style,offset", [("gemma", 1.0), ("llama", 0.0)])
@pytest.mark.parametrize("M,K", [(2, 64), (33, 256), (17, 512), (11, 1024), (5, 1032), (33, 2560), (256, 4096),
                                 (7, 16384)])
def test_rmsnorm_rows(style, offset, M, K):
    from tbf16 import ops
    g = torch.Generator().manual_seed(M * 3 + K)
    x = (torch.randn(M, K, generator=g) * torch.exp2(torch.randint(-10, 10, (M, 1), generator=g).float())).bfloat16()
    w = (torch.randn(K, generator=g) * 0.1).bfloat16()
    r16, s_inv, r = ops.rmsnorm_rows(x.cuda(), w.cuda(), 1e-6, offset, style, want_r=True)
    r16, s_inv, r = r16.cpu(), s_inv.cpu(), r.cpu()
    _, _, r_ref = orc.rmsnorm_rows(x, w, 1e-6, offset, style)
    assert _within_ulp(r, r_ref)
    assert torch.equal(s_inv, orc.row_scale_fused(r, 15))
    assert torch.equal(r16.view(torch.int16), orc.f16_rn(r.float() / s_inv[:, None]).view(torch.int16))


def test_plain_rmsnorm_matches_rmsnorm_rows():
    """ops.rmsnorm (no fp16 operand written) gives the same bf16 rows as rmsnorm_rows."""
    from tbf16 import ops
    x = (torch.randn(3, 5, 256, generator=torch.Generator().manual_seed(9)) * 7).bfloat16().cuda()
    w = (torch.randn(256, generator=torch.Generator().manual_seed(10)) * 0.1).bfloat16().cuda()
    for style, offset in (("gemma", 1.0), ("llama", 0.0)):
        r = ops.rmsnorm(x, w, 1e-6, offset, style)
        _, _, r2 = ops.rmsnorm_rows(x, w, 1e-6, offset, style, want_r=True)
        assert r.shape == x.shape and torch.equal(r.view(torch.int16), r2.view(torch.int16))


@pytest.mark.parametrize("M", [3, 40, 600])
def test_fused_linears_equal_scaled_linear(M):
    """glu_linear / rmsnorm_linear give scaled_linear's bits on the rows the producer wrote (GEMV up to 4
    rows, the skinny GEMM up to 256, the pair GEMM above)."""
    import inputs
    from tbf16 import ops
    I, H, N = 1024, 512, 768
    gate, up = _gate_up(M, I, M)
    w16, ws = ops.prepare_weight(inputs.gemm_w(N, I, seed=3).cuda())
    b = (torch.randn(N, generator=torch.Generator().manual_seed(4)) * 0.1).bfloat16().cuda()
    g, u = gate.cuda(), up.cuda()
    _, _, h = ops.glu_rows(g, u, "silu", want_h=True)
    y = ops.glu_linear(g, u, w16, ws, b, act="silu")
    assert torch.equal(y.view(torch.int16), ops.scaled_linear(h, w16, ws, b).view(torch.int16))
    x = (torch.randn(M, H, generator=torch.Generator().manual_seed(5)) * 4).bfloat16().cuda()
    nw = (torch.randn(H, generator=torch.Generator().manual_seed(6)) * 0.1).bfloat16().cuda()
    w16b, wsb = ops.prepare_weight(inputs.gemm_w(N, H, seed=7).cuda())
    _, _, r = ops.rmsnorm_rows(x, nw, 1e-6, 1.0, "gemma", want_r=True)
    y2 = ops.rmsnorm_linear(x, nw, w16b, wsb, None, eps=1e-6, offset=1.0, style="gemma")
    assert torch.equal(y2.view(torch.int16), ops.scaled_linear(r, w16b, wsb).view(torch.int16))


def test_fused_rows_reject_bad_input():
    from tbf16 import ops
    g = torch.zeros(2, 12, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ops.glu_rows(g, g, "silu")  # row length not a multiple of 8
    g = torch.zeros(2, 16392, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ops.glu_rows(g, g, "silu")  # longer than TBF16_FUSED_MAX_ROW
    with pytest.raises(RuntimeError):
        ops.glu_rows(g[:, :16], g[:, :16], "relu")


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("M,I", [(7, 8), (64, 4096), (3, 10248)])
def test_glu_bwd_matches_torch_autograd(act, M, I):
    """d_gate, d_up in one pass against torch's autograd of act(g) * u on bf16 tensors on the GPU."""
    import torch.nn.functional as F
    from tbf16 import ops
    gate, up = _gate_up(M, I, 3 * M + I)
    g, u = gate.cuda().requires_grad_(), up.cuda().requires_grad_()
    dh = (torch.randn(M, I, generator=torch.Generator().manual_seed(M)) * 0.01).bfloat16().cuda()
    h = (F.silu(g) if act == "silu" else F.gelu(g, approximate="tanh")) * u
    h.backward(dh)
    dg, du = ops.glu_bwd(dh, g.detach(), u.detach(), act)
    for ours, ref in ((dg, g.grad), (du, u.grad)):
        assert _within_ulp(ours.cpu(), ref.cpu())
        assert (ours.view(torch.int16) == ref.view(torch.int16)).float().mean().item() > 0.999


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
def test_glu_linear_training_matches_unfused(act):
    """GLULinearFn (fused rows forward, fused activation backward) against the unfused composition
    act(gate) * up -> autograd.linear: the same scaled GEMMs on operands scaled by the fused and the
    small-kernel rule respectively, so outputs and gradients agree to the fp16 operand rounding."""
    import torch.nn.functional as F
    from helpers import rel_err
    from tbf16 import autograd
    torch.manual_seed(0)
    M, H, I = 512, 256, 1024
    gate = (torch.randn(M, I, device="cuda") * 2).bfloat16().requires_grad_()
    up = torch.randn(M, I, device="cuda").bfloat16().requires_grad_()
    w = (torch.randn(H, I, device="cuda") * 0.03).bfloat16().requires_grad_()
    b = torch.randn(H, device="cuda").bfloat16().requires_grad_()
    dy = torch.randn(M, H, device="cuda").bfloat16()
    y = autograd.glu_linear(gate, up, w, b, act)
    y.backward(dy)
    got = [y.detach(), gate.grad, up.grad, w.grad, b.grad]
    for t in (gate, up, w, b):
        t.grad = None
    a = F.silu(gate) if act == "silu" else F.gelu(gate, approximate="tanh")
    y2 = autograd.linear(a * up, w, b)
    y2.backward(dy)
    ref = [y2.detach(), gate.grad, up.grad, w.grad, b.grad]
    for name, x, r in zip(("y", "d_gate", "d_up", "dW", "db"), got, ref):
        assert torch.isfinite(x.float()).all(), name
        assert rel_err(x, r) < 5e-3, (name, rel_err(x, r))


def _rope_ref(y, cos, sin):
    """The model-side rotary embedding on bf16 tensors (rotate-half)."""
    D = y.shape[-1]
    rot = torch.cat([-y[..., D // 2:], y[..., :D // 2]], -1)
    return y * cos + rot * sin


@pytest.mark.parametrize("D", [64, 128, 256, 512])
@pytest.mark.parametrize("norm", [True, False])
def test_rmsnorm_rope_matches_torch(D, norm):
    """QK-norm + RoPE in one pass: bit-equal to torch's bf16 ops on the same normed rows (the norm itself
    is rmsnorm_rows' arithmetic, checked against the oracle above)."""
    from tbf16 import ops
    g = torch.Generator().manual_seed(D + norm)
    B, S, H = 2, 37, 3
    x = (torch.randn(B, S, H, D, generator=g) * torch.exp2(torch.randint(-6, 6, (B, S, H, 1), generator=g).float()))
    x = x.bfloat16().cuda()
    w = (torch.randn(D, generator=g) * 0.2).bfloat16().cuda() if norm else None
    pos = torch.arange(S, dtype=torch.float32)
    inv = 1.0 / (1e4 ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    ang = torch.outer(pos, inv)
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16().cuda()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16().cuda()
    out = ops.rmsnorm_rope(x, w, cos[None, None], sin[None, None], 1e-6, 1.0, "gemma")
    y = ops.rmsnorm(x, w, 1e-6, 1.0, "gemma") if norm else x
    ref = _rope_ref(y.transpose(1, 2), cos, sin).transpose(1, 2)  # the model applies it on (B, H, S, D)
    assert out.shape == x.shape
    assert torch.equal(out.view(torch.int16), ref.contiguous().view(torch.int16))


def test_rmsnorm_rope_rejects():
    from tbf16 import ops
    x = torch.zeros(1, 4, 2, 96, dtype=torch.bfloat16, device="cuda")
    c = torch.zeros(4, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError):
        ops.rmsnorm_rope(x, None, c, c)  # D = 96 is not one of 64, 128, 256, 512
    with pytest.raises(RuntimeError):
        ops.rmsnorm_rope(x[..., :64], None, c[:3, :64], c[:3, :64])  # cos / sin for the wrong S


def test_rmsnorm_rope_column_slices_of_fused_qkv():
    """q and k read in place as column slices of one [tokens, (Hq + 2 Hkv) D] projection output."""
    from tbf16 import ops
    g = torch.Generator().manual_seed(5)
    B, S, Hq, Hk, D = 2, 19, 4, 2, 128
    qkv = (torch.randn(B, S, (Hq + 2 * Hk) * D, generator=g) * 3).bfloat16().cuda()
    q = qkv[..., :Hq * D].view(B, S, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hk) * D].view(B, S, Hk, D)
    ang = torch.outer(torch.arange(S, dtype=torch.float32), 1.0 / (1e4 ** (torch.arange(0, D, 2) / D)))
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16().cuda()
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16().cuda()
    for t, seed in ((q, 1), (k, 2)):
        w = (torch.randn(D, generator=torch.Generator().manual_seed(seed)) * 0.2).bfloat16().cuda()
        out = ops.rmsnorm_rope(t, w, cos, sin)
        ref = ops.rmsnorm_rope(t.contiguous(), w, cos, sin)
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        ref2 = _rope_ref(ops.rmsnorm(t.contiguous(), w, 1e-6, 1.0, "gemma").transpose(1, 2), cos, sin).transpose(1, 2)
        assert torch.equal(out.view(torch.int16), ref2.contiguous().view(torch.int16))


@pytest.mark.parametrize("M,K", [(5, 256), (2048, 2560), (1100, 4096), (3, 10240)])
def test_residual_norm_forms(M, K):
    """x + rmsnorm(y) and (s = residual + [rmsnorm](x), rmsnorm_rows(s)) in one pass each: bit-equal to the
    unfused sequence of ops.rmsnorm / torch's bf16 add / rmsnorm_rows (warp-per-row and block shapes)."""
    from tbf16 import ops
    g = torch.Generator().manual_seed(M + K)
    x = (torch.randn(M, K, generator=g) * 4).bfloat16().cuda()
    res = (torch.randn(M, K, generator=g) * 30).bfloat16().cuda()
    w = (torch.randn(K, generator=g) * 0.1).bfloat16().cuda()
    pw = (torch.randn(K, generator=g) * 0.1).bfloat16().cuda()
    eq = lambda a, b: torch.equal(a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))
    assert eq(ops.rmsnorm(x, pw, residual=res), res + ops.rmsnorm(x, pw))
    for post in (pw, None):
        s, r16, s_inv = ops.add_rmsnorm_rows(x, res, w, post_weight=post)
        s_ref = res + (ops.rmsnorm(x, post) if post is not None else x)
        r16_ref, s_inv_ref = ops.rmsnorm_rows(s_ref, w)
        assert eq(s, s_ref) and eq(r16, r16_ref) and torch.equal(s_inv, s_inv_ref)
