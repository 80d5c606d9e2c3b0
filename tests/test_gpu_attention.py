"""Parity of the tcgen05 scaled-attention forward with the oracle (reference attention.py:38-65 restated
in fp64 from the exact fp16 operands): integer exponents bit-exact, outputs within one bf16 ulp plus
the fp16 rounding of P (2^-10 of the head's V scale), and within 2e-3 relative of fp64, including
Q/K whose raw logits overflow fp16. Called through tbf16.attention (ctypes -> C ABI)."""
import math

import pytest
import torch

import inputs
from helpers import bf16_ulp, rel_err
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _check_out(out, q, k, v, causal, mask=None, scale=None, v_exp=13):
    f = orc.sdpa_fwd(q.cpu(), k.cpu(), v.cpu(), attn_mask=None if mask is None else mask.cpu(), is_causal=causal,
                     scale=scale, v_exp=v_exp)
    ref = f["out"]
    H = q.shape[1]
    vmax = orc._expand_kv(v.cpu().double().abs().amax(dim=(-2, -1), keepdim=True), H)
    d = (out.cpu().double() - ref.double()).abs()
    # one bf16 ulp + the fp16 rounding of P (2^-11 relative, doubled) + the fp32 rounding of the logits
    # themselves (4 ulp of the row's largest scaled logit moves each softmax weight by that much relative;
    # it matters only for near-ties under logits that overflow fp16, as in config 3)
    two_ev = torch.ldexp(torch.ones(()), orc.expand_heads(f["ev"], H).double())[..., None, None]
    logit_err = 2.0 ** -21 * f["zmax"][..., None] * (f["pv_abs"] + f["o16"].abs()) * two_ev
    tol = bf16_ulp(ref) + 2.0 ** -10 * vmax + logit_err
    bad = d > tol
    assert not bad.any(), f"{int(bad.sum())} elements outside tolerance (max excess {(d - tol)[bad].max():.3e})"
    exact = f["o16"] * torch.ldexp(torch.ones(()), orc.expand_heads(f["ev"], H).double())[..., None, None]
    assert rel_err(out, exact) < 2e-3
    assert torch.isfinite(out.float()).all()
    return f


@pytest.mark.parametrize("B,H,Hkv,S,D,causal", [(1, 2, 2, 128, 64, False), (1, 2, 2, 256, 128, True),
                                                (2, 4, 2, 200, 128, False), (1, 4, 1, 333, 64, True),
                                                (1, 16, 16, 1024, 128, True), (2, 2, 2, 96, 128, True),
                                                # more 256-row items than SMs: the persistent two-tile kernel
                                                # (fewer go to the one-tile kernel), ragged lengths included
                                                (4, 40, 8, 333, 128, True), (3, 64, 64, 200, 64, False),
                                                (2, 48, 16, 520, 128, False)])
def test_sdpa_forward_vs_oracle(B, H, Hkv, S, D, causal):
    from tbf16 import attention
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=S + H, Hkv=Hkv)  # raw logits overflow fp16
    out = attention.sdpa(q.cuda(), k.cuda(), v.cuda(), is_causal=causal, enable_gqa=Hkv != H)
    _check_out(out, q, k, v, causal)


def test_sdpa_exponents_and_operands_bit_exact():
    from tbf16 import attention
    q, k, v = inputs.attention_qkv(1, 4, 192, 64, seed=3, qk_exp=12)
    q16, k16, v16, a, ev = attention.prepare_qkv(q.cuda(), k.cuda(), v.cuda(), v_exp=13)
    rq, rk, rv, ra, rev = orc.prepare_qkv(q, k, v, 13)
    assert int(a) == int(ra) and torch.equal(ev.cpu(), rev)
    for x, y in ((q16, rq), (k16, rk), (v16, rv)):
        assert torch.equal(x.cpu().view(torch.int16), y.view(torch.int16))


def test_sdpa_cross_lengths_and_masks():
    """Sq != Sk, a broadcast bool padding mask and an additive bf16 mask (diffusers-style calls)."""
    from tbf16 import attention
    B, H, Sq, Sk, D = 2, 4, 160, 300, 64
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, H, Sq, D, generator=g).bfloat16()
    k = torch.randn(B, H, Sk, D, generator=g).bfloat16()
    v = torch.randn(B, H, Sk, D, generator=g).bfloat16()
    keep = torch.ones(B, Sk, dtype=torch.bool)
    keep[:, Sk * 2 // 3:] = False
    for mask in (keep[:, None, None, :], (~keep).to(torch.bfloat16)[:, None, None, :] * -10000.0):
        out = attention.sdpa(q.cuda(), k.cuda(), v.cuda(), attn_mask=mask.cuda())
        _check_out(out, q, k, v, False, mask=mask)


@pytest.mark.parametrize("B,H,Hkv,S,causal", [(1, 8, 4, 2048, True), (2, 2, 1, 333, False)])
def test_sdpa_head_dim_256(B, H, Hkv, S, causal):
    """Gemma-3-shaped attention (head dim 256, GQA 8/4, causal prefill) through the D=256 kernel."""
    from tbf16 import attention
    q, k, v = inputs.attention_qkv(B, H, S, 256, seed=S + 256, Hkv=Hkv, qk_exp=4)
    out = attention.sdpa(q.cuda(), k.cuda(), v.cuda(), is_causal=causal, enable_gqa=Hkv != H)
    _check_out(out, q, k, v, causal)


def test_sdpa_head_dim_padding():
    """Head dims that are not 64/128/256 are zero-padded (logits unchanged) and sliced back."""
    from tbf16 import attention
    for D in (32, 112, 200):
        q, k, v = inputs.attention_qkv(1, 2, 130, D, seed=D)
        out = attention.sdpa(q.cuda(), k.cuda(), v.cuda())
        assert out.shape == (1, 2, 130, D)
        _check_out(out, q, k, v, False)


def test_sdpa_permuted_inputs():
    from tbf16 import attention
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(2, 256, 8, 64, generator=g).mul(3e3).bfloat16().permute(0, 2, 1, 3) for _ in range(3))
    out = attention.sdpa(q.cuda(), k.cuda(), v.cuda())
    _check_out(out, q.contiguous(), k.contiguous(), v.contiguous(), False)


def test_sdpa_config3_16k_properties():
    """Config 3 at full size (B=1, H=16, D=128, S=16384): finite, and sampled rows against fp64."""
    from tbf16 import attention
    B, H, S, D = 1, 16, 16384, 128
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=0, device="cuda")
    for causal in (False, True):
        out = attention.sdpa(q, k, v, is_causal=causal)
        assert torch.isfinite(out.float()).all()
        rows = torch.tensor([0, 1, 777, 8191, 16383])
        for h in (0, 7, 15):
            qs = q[0, h, rows].double().cpu()
            s = qs @ k[0, h].double().cpu().t() / math.sqrt(D)
            if causal:
                s = s.masked_fill(torch.arange(S)[None, :] > rows[:, None], float("-inf"))
            ref = torch.softmax(s, -1) @ v[0, h].double().cpu()
            assert rel_err(out[0, h, rows].cpu(), ref) < 2e-3


def test_lse_output():
    from tbf16 import attention
    q, k, v = inputs.attention_qkv(1, 2, 256, 128, seed=8)
    q16, k16, v16, a, ev = attention.prepare_qkv(q.cuda(), k.cuda(), v.cuda(), v_exp=0)
    out, lse = attention.attn_forward(q16, k16, v16, ev, is_causal=True, need_lse=True)
    f = orc.sdpa_fwd(q, k, v, is_causal=True, v_exp=0)
    assert lse.shape[-1] % 128 == 0  # padded row stride for the backward's bulk copies
    assert torch.allclose(lse[..., :256].cpu().double(), f["lse"], rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("D", [128, 256])
def test_sdpa_output_in_token_major_order(D):
    """Inference output is (B, H, S, D) over (B, S, H, D) memory (as torch's own SDPA returns it), so the
    model's transpose + reshape for the output projection is a view; values equal the contiguous call."""
    from tbf16 import attention, _ext
    torch.manual_seed(0)
    B, H, Hkv, S = 2, 4, 2, 300
    q = torch.randn(B, H, S, D, device="cuda").bfloat16()
    k = torch.randn(B, Hkv, S, D, device="cuda").bfloat16()
    v = torch.randn(B, Hkv, S, D, device="cuda").bfloat16()
    out = attention.sdpa(q, k, v, is_causal=True, enable_gqa=True)
    assert out.shape == (B, H, S, D) and out.transpose(1, 2).is_contiguous()
    q16, k16, v16, _, ev = attention.prepare_qkv(q, k, v, v_exp=13)
    ref = torch.empty(B, H, S, D, device="cuda", dtype=torch.bfloat16)
    _ext.call("tbf16_attn_fwd", _ext.ptr(q16), _ext.ptr(k16), _ext.ptr(v16), B, H, Hkv, S, S, D, 1.0 / D ** 0.5, 1,
              _ext.ptr(ev.contiguous()), None, 0, 0, 0, _ext.ptr(ref), None, 0, None, _ext.stream_ptr(q.device))
    assert torch.equal(out.contiguous().view(torch.int16), ref.view(torch.int16))
