"""Attention dropout (the reference passes dropout_p to torch's memory-efficient attention,
tbf16/autograd.py:159-160,179-181; tbf16/attention.py:63-64). This build draws its mask from a
counter-based hash of (seed, batch*head, query, key), so masks are not torch's Philox stream; what must
hold is that (1) the GPU's mask is the documented function of its inputs (checked bit for bit against the
oracle's restatement) with the requested keep rate, and (2) given that mask, forward and gradients are
those of softmax(S) * mask / keep_probability @ V (checked against fp64 autograd, 2e-3 relative), and the
backward uses the forward's mask."""
import ctypes
import math

import pytest
import torch

from helpers import rel_err, report
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _keep_gpu(seed, BH, Sq, Sk, p):
    from tbf16 import _ext
    keep = torch.empty(BH, Sq, Sk, dtype=torch.uint8, device="cuda")
    _ext.call("tbf16_attn_dropout_keep", _ext.ptr(keep), BH, Sq, Sk, float(p), ctypes.c_uint64(seed), _ext.stream_ptr())
    return keep.bool()


@pytest.mark.parametrize("p", [0.1, 0.5])
def test_dropout_mask_matches_restatement_and_rate(p):
    seed = 0x1234_5678_9ABC_DEF0
    keep = _keep_gpu(seed, 6, 300, 257, p)
    ref = orc.dropout_keep(seed, 6, 300, 257, p)
    assert torch.equal(keep.cpu(), ref)
    n = keep.numel()
    thr, _ = orc.dropout_params(p)
    q = (65536 - thr) / 65536
    assert abs(keep.float().mean().item() - q) < 5 * math.sqrt(q * (1 - q) / n)
    assert not torch.equal(_keep_gpu(seed + 1, 6, 300, 257, p), keep)


def _masked_attention(q, k, v, keep, causal, scale, inv_keep):
    """fp64 softmax(q k^T * scale) with dropped weights zeroed and kept ones scaled, @ v (GQA expanded)."""
    H = q.shape[1]
    if k.shape[1] != H:
        k = k.repeat_interleave(H // k.shape[1], 1)
        v = v.repeat_interleave(H // v.shape[1], 1)
    s = (q @ k.transpose(-1, -2)) * scale
    if causal:
        S = s.shape[-1]
        s = s.masked_fill(torch.ones(s.shape[-2], S, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    pm = torch.softmax(s, -1) * keep.to(s.dtype) * inv_keep
    return pm @ v


@pytest.mark.parametrize("B,Hq,Hkv,S,D,causal,p", [(1, 4, 4, 512, 64, True, 0.1), (2, 4, 2, 384, 128, False, 0.3),
                                                   (1, 4, 2, 333, 128, True, 0.5), (1, 2, 2, 256, 256, True, 0.2)])
def test_dropout_forward_backward_vs_fp64(B, Hq, Hkv, S, D, causal, p):
    from tbf16 import autograd as ag
    g = torch.Generator().manual_seed(S + D)
    q = torch.randn(B, Hq, S, D, generator=g).bfloat16().cuda()
    k = torch.randn(B, Hkv, S, D, generator=g).bfloat16().cuda()
    v = torch.randn(B, Hkv, S, D, generator=g).bfloat16().cuda()
    do = torch.randn(B, Hq, S, D, generator=g).bfloat16().cuda()
    ins = [t.detach().clone().requires_grad_() for t in (q, k, v)]
    torch.manual_seed(7)
    seed = torch.randint(0, 1 << 32, (2,), dtype=torch.int64).tolist()  # what dropout_seed draws next
    torch.manual_seed(7)
    out = ag.sdpa(*ins, dropout_p=p, is_causal=causal, enable_gqa=Hq != Hkv)
    out.backward(do)
    seed = (seed[1] << 32) | seed[0]
    _, inv_keep = orc.dropout_params(p)
    keep = _keep_gpu(seed, B * Hq, S, S, p).view(B, Hq, S, S)
    ex = [t.detach().double().requires_grad_() for t in (q, k, v)]
    o64 = _masked_attention(*ex, keep, causal, 1.0 / math.sqrt(D), inv_keep)
    o64.backward(do.double())
    errs = {"o": rel_err(out, o64), "dq": rel_err(ins[0].grad, ex[0].grad), "dk": rel_err(ins[1].grad, ex[1].grad),
            "dv": rel_err(ins[2].grad, ex[2].grad)}
    report(f"dropout p={p} B={B} H={Hq}/{Hkv} S={S} D={D} causal={causal} vs fp64", **errs)
    for t in (out, ins[0].grad, ins[1].grad, ins[2].grad):
        assert torch.isfinite(t.float()).all()
    for what, e in errs.items():
        assert e < 2e-3, (what, e)


def test_dropout_zero_is_the_plain_path():
    from tbf16 import attention
    q, k, v = (torch.randn(1, 2, 200, 64, device="cuda").bfloat16() for _ in range(3))
    a = attention.sdpa(q, k, v, is_causal=True)
    b = attention.sdpa(q, k, v, is_causal=True, dropout_p=0.0)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
