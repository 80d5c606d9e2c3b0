"""Key-split schedule of the head-dim-256 attention forward (tbf16_attn_fwd_ws): shapes with few 256-row
query blocks for the device's CTA pairs cut their longest blocks into two parts over the key tiles, run
by different pairs and added through the workspace. Parity with the oracle (reference attention.py:38-65
restated in fp64) at the same bound as the plain schedule, the schedule actually taken (workspace size
> 0), lse / o16 / dropout / masks through the combine, and a workspace too small for the plan running
the plain schedule bit for bit. Called through the C ABI."""
import pytest
import torch

import inputs
from helpers import bf16_ulp, rel_err
from oracle import oracle as orc
from test_gpu_attention import _check_out

pytestmark = pytest.mark.gpu

D = 256


def _ws_size(B, H, Hkv, Sq, Sk, causal):
    from tbf16 import _ext
    return int(_ext.lib().tbf16_attn_fwd_ws_size(B, H, Hkv, Sq, Sk, D, int(causal)))


def _prep(q, k, v, v_exp=13):
    from tbf16 import attention
    return attention.prepare_qkv(q.cuda(), k.cuda(), v.cuda(), v_exp=v_exp)


def _fwd(q16, k16, v16, ev, causal, ws_bytes=None, mask=None, lse=False, o16=False, dropout_p=0.0, seed=0):
    """One forward through tbf16_attn_fwd_ws; ws_bytes None: the plan's size, 0: no workspace."""
    from tbf16 import _ext
    from tbf16.attention import additive_mask
    B, H, Sq, _ = q16.shape
    Hkv, Sk = k16.shape[1], k16.shape[2]
    need = _ws_size(B, H, Hkv, Sq, Sk, causal)
    nb = need if ws_bytes is None else ws_bytes
    ws = torch.empty(max(nb, 16), device="cuda", dtype=torch.uint8)
    out = torch.empty(B, H, Sq, D, device="cuda", dtype=torch.bfloat16)
    ld = (Sq + 127) // 128 * 128
    lse_t = torch.empty(B, H, ld, device="cuda", dtype=torch.float32) if lse else None
    o16_t = torch.empty(B, H, Sq, D, device="cuda", dtype=torch.float16) if o16 else None
    m = additive_mask(mask, B, H, Sq, Sk, q16.device) if mask is not None else None
    ms = m.stride()[:3] if m is not None else (0, 0, 0)
    _ext.call("tbf16_attn_fwd_ws", _ext.ptr(q16), _ext.ptr(k16), _ext.ptr(v16), B, H, Hkv, Sq, Sk, D, D ** -0.5,
              int(causal), _ext.ptr(ev.contiguous()), _ext.ptr(m), *ms, _ext.ptr(out), *out.stride()[:3],
              _ext.ptr(lse_t), ld, _ext.ptr(o16_t), float(dropout_p), int(seed), _ext.ptr(ws) if nb else None, nb,
              _ext.stream_ptr(q16.device))
    torch.cuda.synchronize()
    return out, lse_t, o16_t


@pytest.mark.parametrize("B,H,Hkv,S,causal", [(1, 8, 4, 2048, True), (1, 2, 1, 4096, True), (1, 1, 1, 2900, True),
                                              (1, 1, 1, 2048, False)])
def test_split_vs_oracle(B, H, Hkv, S, causal):
    assert _ws_size(B, H, Hkv, S, S, causal) > 0, "shape expected to take the key-split schedule"
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=S + H, Hkv=Hkv, qk_exp=4)
    q16, k16, v16, _, ev = _prep(q, k, v)
    out, _, _ = _fwd(q16, k16, v16, ev, causal)
    _check_out(out, q, k, v, causal)


def test_split_cross_lengths_ragged():
    """Sq != Sk, neither a multiple of the tile: 2 query blocks over 24 key tiles, the last one partial."""
    B, H, Sq, Sk = 1, 1, 300, 3000
    assert _ws_size(B, H, H, Sq, Sk, False) > 0
    g = torch.Generator().manual_seed(21)
    q = (torch.randn(B, H, Sq, D, generator=g) * 16).bfloat16()
    k = (torch.randn(B, H, Sk, D, generator=g) * 16).bfloat16()
    v = (torch.randn(B, H, Sk, D, generator=g) * 64).bfloat16()
    q16, k16, v16, _, ev = _prep(q, k, v)
    out, _, _ = _fwd(q16, k16, v16, ev, False)
    _check_out(out, q, k, v, False)


def test_split_with_mask():
    """A mask hiding the second half of the keys: the later parts see only masked logits for those rows
    (running max -inf), and the combine must give them weight zero."""
    B, H, S = 1, 2, 1536
    assert _ws_size(B, H, H, S, S, False) > 0
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=33, qk_exp=4)
    keep = torch.ones(B, S, dtype=torch.bool)
    keep[:, S // 2:] = False
    mask = keep[:, None, None, :]
    q16, k16, v16, _, ev = _prep(q, k, v)
    out, _, _ = _fwd(q16, k16, v16, ev, False, mask=mask.cuda())
    _check_out(out, q, k, v, False, mask=mask)


def test_split_lse_and_o16():
    """The training forward's extra outputs come from the combined parts: lse against fp64, o16 against
    the plain schedule's within the fp16 rounding of P."""
    B, H, S = 1, 2, 1800
    assert _ws_size(B, H, H, S, S, False) > 0
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=44, qk_exp=4)
    q16, k16, v16, _, ev = _prep(q, k, v, v_exp=0)
    out, lse, o16 = _fwd(q16, k16, v16, ev, False, lse=True, o16=True)
    _, lse_p, o16_p = _fwd(q16, k16, v16, ev, False, ws_bytes=0, lse=True, o16=True)
    f = orc.sdpa_fwd(q, k, v, is_causal=False, v_exp=0)
    assert torch.allclose(lse[..., :S].cpu().double(), f["lse"], rtol=1e-5, atol=1e-4)
    assert torch.allclose(lse, lse_p, rtol=1e-6, atol=1e-5)
    vmax = v16.float().abs().amax(dim=(-2, -1), keepdim=True)
    assert ((o16.float() - o16_p.float()).abs() <= 2.0 ** -9 * vmax + bf16_ulp(o16_p.float())).all()
    assert rel_err(o16.cpu(), f["o16"]) < 2e-3


def test_split_dropout_matches_plain():
    """The dropout mask depends on (seed, head, query, key) only: split and plain schedules drop the same
    weights, so their outputs agree within the fp16 rounding of P."""
    B, H, S = 1, 2, 4096
    assert _ws_size(B, H, H, S, S, True) > 0
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=55, qk_exp=4, device="cuda")
    q16, k16, v16, _, ev = _prep(q, k, v)
    a, _, _ = _fwd(q16, k16, v16, ev, True, dropout_p=0.2, seed=1234)
    b, _, _ = _fwd(q16, k16, v16, ev, True, ws_bytes=0, dropout_p=0.2, seed=1234)
    scale = torch.ldexp(torch.ones((), device="cuda"), ev.float().amax())
    vmax = v16.float().abs().amax() * scale / 0.8
    d = (a.float() - b.float()).abs()
    assert (d <= bf16_ulp(b.float()) * 2 + 2.0 ** -9 * vmax).all()
    assert torch.isfinite(a.float()).all()


def test_split_small_workspace_runs_plain_schedule():
    """A workspace smaller than the plan (or none) leaves the plain schedule: bit-equal outputs."""
    B, H, Hkv, S = 1, 8, 4, 2048
    need = _ws_size(B, H, Hkv, S, S, True)
    assert need > 0
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=66, Hkv=Hkv, qk_exp=4, device="cuda")
    q16, k16, v16, _, ev = _prep(q, k, v)
    a, _, _ = _fwd(q16, k16, v16, ev, True, ws_bytes=need - 16)
    b, _, _ = _fwd(q16, k16, v16, ev, True, ws_bytes=0)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_split_schedule_only_for_few_items():
    """Shapes that fill the pairs, shapes whose split would not pay, and head dims below 256 keep the plain
    schedule and need no workspace."""
    assert _ws_size(1, 16, 16, 8192, 8192, True) == 0
    assert _ws_size(4, 8, 4, 2048, 2048, True) == 0
    assert _ws_size(1, 8, 4, 1024, 1024, True) == 0
    from tbf16 import _ext
    assert int(_ext.lib().tbf16_attn_fwd_ws_size(1, 8, 4, 2048, 2048, 128, 1)) == 0


def test_split_graph_replays():
    """Tickets and flags are zeroed by each launch (a memset node in a captured graph), and the combine
    gives the same bits whichever part finishes first: replays give the eager call's output exactly."""
    from tbf16 import attention
    B, H, Hkv, S = 1, 8, 4, 2048
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=77, Hkv=Hkv, qk_exp=4, device="cuda")
    ref = attention.sdpa(q, k, v, is_causal=True, enable_gqa=True).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        attention.sdpa(q, k, v, is_causal=True, enable_gqa=True)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = attention.sdpa(q, k, v, is_causal=True, enable_gqa=True)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
