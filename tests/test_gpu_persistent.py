"""The persistent attention forward kernels walk several work items per CTA (head dims 64 / 128: pairs of
128-row query tiles, one CTA per SM) or per CTA pair (head dim 256: 256 query rows, one pair per two
SMs), with their K/V rings, S buffers and barrier phases running on across items. These cases give
every CTA more than one item, ragged last items, GQA, Sq != Sk and a single query row, and check the
output and the logsumexp against the oracle (reference attention.py:38-65 restated in fp64) with the
same bounds as test_gpu_attention.py, plus bit-for-bit agreement of repeated calls."""
import math

import pytest
import torch

import inputs
from oracle import oracle as orc
from test_gpu_attention import _check_out

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("causal", [False, True])
def test_many_items_per_cta(D, causal):
    """B=3, 20 query heads over 5 KV heads, S=700: 180 items of 256 rows (2.4 per CTA pair at D=256),
    360 two-tile items at D <= 128 (2.4 per CTA), the last of each head ragged."""
    from tbf16 import attention
    B, H, Hkv, S = 3, 20, 5, 700
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=D + int(causal), Hkv=Hkv, qk_exp=4)
    outs = [attention.sdpa(q.cuda(), k.cuda(), v.cuda(), is_causal=causal, enable_gqa=True) for _ in range(2)]
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    _check_out(outs[0], q, k, v, causal)


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("Sq,Sk", [(1000, 300), (300, 1000), (1, 517)])
@pytest.mark.parametrize("causal", [False, True])
def test_cross_lengths(D, Sq, Sk, causal):
    """Sq != Sk (top-left causal alignment, as torch's is_causal) and a single query row."""
    from tbf16 import attention
    g = torch.Generator().manual_seed(Sq * 7 + Sk + D)
    q = (torch.randn(2, 4, Sq, D, generator=g) * 8).bfloat16()
    k = (torch.randn(2, 4, Sk, D, generator=g) * 8).bfloat16()
    v = (torch.randn(2, 4, Sk, D, generator=g) * 3).bfloat16()
    out = attention.sdpa(q.cuda(), k.cuda(), v.cuda(), is_causal=causal)
    _check_out(out, q, k, v, causal)


@pytest.mark.parametrize("D", [128, 256])
def test_lse_and_o16_many_items(D):
    """The training outputs of the persistent kernels (natural-log lse per row, fp16 O before the V
    scale) over many items per CTA: lse as close to the oracle's as test_gpu_attention.py asks (fp32 row
    max and row sum), O16 within one fp16 ulp plus P's fp16 rounding."""
    from tbf16 import attention
    B, H, S = 2, 24, 600
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=3 + D, qk_exp=0)
    q16, k16, v16, a, ev = attention.prepare_qkv(q.cuda(), k.cuda(), v.cuda())
    out, lse, o16 = attention.attn_forward(q16, k16, v16, ev, None, True, 1.0 / math.sqrt(D), need_lse=True,
                                           need_o16=True)
    f = orc.sdpa_fwd(q, k, v, is_causal=True, v_exp=0)
    assert torch.allclose(lse[..., :S].cpu().double(), f["lse"], rtol=1e-5, atol=1e-4)
    o_ref = f["o16"]
    vmax = orc._expand_kv(f["v16"].double().abs().amax(dim=(-2, -1), keepdim=True), H)
    err = (o16.cpu().double() - o_ref).abs()
    tol = 2.0 ** -10 * o_ref.abs() + 2.0 ** -10 * vmax
    assert (err <= tol).all(), float((err - tol).max())
