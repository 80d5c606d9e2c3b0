"""bf16 scaled_dot_product_attention on fp16 tensor cores, B200 kernels.

Same public surface as the reference's tbf16/attention.py. Q is multiplied by 2**a and K by 2**-a,
which leaves every logit unchanged, with `a` chosen so both fit fp16's range. V gets one power-of-two
scale per (batch, head), undone on the output. All scales are exact powers of two computed on the
GPU (no host sync) by tbf16_prepare_qkv; the attention itself is this build's tcgen05 flash-attention
kernel, which writes bf16 straight from its fp32 accumulator.

Limit (as in the reference): amax(|q|) * amax(|k|) < 2**28, i.e. raw logits below ~2.7e8 before the
softmax scale.
"""
import math

import torch

from ._ext import BF16, F16, call, lib, ptr, require_cuda, stream_ptr

_DTYPE = {torch.bfloat16: BF16, torch.float16: F16}
KERNEL_D = (64, 128, 256)      # forward kernel head dims (others are zero-padded up)
KERNEL_D_TRAIN = (64, 128, 256)  # backward kernel head dims


def _fast(x: torch.Tensor):
    """Kept from the reference (attention.py:18-21): whether a tensor meets the kernels' layout needs."""
    return (x.is_cuda and x.dim() == 4 and x.stride(-1) == 1 and x.shape[-1] % 8 == 0 and x.data_ptr() % 16 == 0
            and all(s % 8 == 0 for s in x.stride()[:3]) and x.dtype in _DTYPE)


def _as_kernel_layout(x):
    require_cuda(x)
    if x.dtype not in _DTYPE:
        raise RuntimeError(f"tbf16 attention: bf16 or fp16 tensors expected, got {x.dtype}")
    if not _fast(x):
        x = x.contiguous()
        if x.shape[-1] % 8:
            x = torch.nn.functional.pad(x, (0, 8 - x.shape[-1] % 8))
    return x


def head_exp(x: torch.Tensor):
    """int32 (B, H): e with amax(|x[b, h]|) = m * 2**e, m in [0.5, 1) (0 for all-zero heads)."""
    x = _as_kernel_layout(x)
    B, H, S, D = x.shape
    e = torch.empty((B, H), device=x.device, dtype=torch.int32)
    ws = torch.empty(B * H, device=x.device, dtype=torch.float32)
    call("tbf16_head_exp", ptr(x), _DTYPE[x.dtype], B, H, S, D, *x.stride()[:3], ptr(e), ptr(ws), stream_ptr(x.device))
    return e


def head_scale(x: torch.Tensor, e: torch.Tensor, dtype):
    """x * 2**e[b, h] cast to dtype, as a contiguous (B, H, S, D) tensor. Exact while in range."""
    D0 = x.shape[-1]
    x = _as_kernel_layout(x)
    B, H, S, D = x.shape
    e = e.to(device=x.device, dtype=torch.int32).expand(B, H)
    y = torch.empty((B, H, S, D), device=x.device, dtype=dtype)
    call("tbf16_head_scale_cast", ptr(x), _DTYPE[x.dtype], B, H, S, D, *x.stride()[:3], ptr(e), e.stride(0),
         e.stride(1), ptr(y), _DTYPE[dtype], stream_ptr(x.device))
    return y if D == D0 else y[..., :D0].contiguous()


def prepare_qkv(q, k, v, v_exp=0):
    """Scaled fp16 copies of q, k, v and the exponents to undo them: (q16, k16, v16, a, ev).
    V's per-head max goes to [2^(v_exp-1), 2^v_exp); ev already includes -v_exp."""
    q, k, v = _as_kernel_layout(q), _as_kernel_layout(k), _as_kernel_layout(v)
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise RuntimeError("tbf16.prepare_qkv: bf16 q, k, v expected")
    B, Hq, Sq, D = q.shape
    Bk, Hkv, Sk, Dk = k.shape
    if Bk != B or Dk != D or v.shape != k.shape or Hq % Hkv:
        raise RuntimeError(f"tbf16.prepare_qkv: incompatible shapes {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    dev = q.device
    q16 = torch.empty((B, Hq, Sq, D), device=dev, dtype=torch.float16)
    k16 = torch.empty((B, Hkv, Sk, D), device=dev, dtype=torch.float16)
    v16 = torch.empty((B, Hkv, Sk, D), device=dev, dtype=torch.float16)
    a = torch.empty((), device=dev, dtype=torch.int32)
    ev = torch.empty((B, Hkv), device=dev, dtype=torch.int32)
    ws = torch.empty(B * Hq + 2 * B * Hkv, device=dev, dtype=torch.float32)
    call("tbf16_prepare_qkv", ptr(q), *q.stride()[:3], ptr(k), *k.stride()[:3], ptr(v), *v.stride()[:3], B, Hq, Hkv, Sq,
         Sk, D, int(v_exp), ptr(q16), ptr(k16), ptr(v16), ptr(a), ptr(ev), ptr(ws), stream_ptr(dev))
    return q16, k16, v16, a, ev


def expand_heads(e, n_heads):
    """Per-KV-head exponents -> per-query-head (GQA)."""
    return e if e.shape[1] == n_heads else e.repeat_interleave(n_heads // e.shape[1], dim=1)


def additive_mask(attn_mask, B, H, Sq, Sk, device):
    """attn_mask -> fp16 additive bias broadcastable to (B, H, Sq, Sk) with a contiguous key dimension;
    boolean masks become 0 / -inf, float masks are cast to fp16 as the reference does
    (attention.py:61-62; large negatives become -inf)."""
    if attn_mask is None:
        return None
    m = attn_mask
    if m.dtype == torch.bool:
        m = torch.zeros(m.shape, dtype=torch.float16, device=device).masked_fill_(~m.to(device), float("-inf"))
    else:
        m = m.to(device=device, dtype=torch.float16)
    while m.dim() < 4:
        m = m.unsqueeze(0)
    m = m.expand(B, H, Sq, Sk)
    if m.stride(-1) != 1:
        m = m.contiguous()
    return m


def dropout_seed() -> int:
    """A 64-bit seed for the attention dropout mask, drawn from torch's default CPU generator (so
    torch.manual_seed makes the masks reproducible)."""
    lo, hi = torch.randint(0, 1 << 32, (2,), dtype=torch.int64).tolist()
    return (hi << 32) | lo


_FWD_WS = {}


def _fwd_ws_size(B, Hq, Hkv, Sq, Sk, D, causal):
    """Workspace bytes of the key-split head-dim-256 forward for this shape (0: plain schedule)."""
    key = (B, Hq, Hkv, Sq, Sk, D, causal, torch.cuda.current_device())
    n = _FWD_WS.get(key)
    if n is None:
        n = _FWD_WS[key] = int(lib().tbf16_attn_fwd_ws_size(B, Hq, Hkv, Sq, Sk, D, int(causal))) if D == 256 else 0
    return n


def attn_forward(q16, k16, v16, ev, attn_mask=None, is_causal=False, scale=None, d_orig=None, need_lse=False,
                 need_o16=False, dropout_p=0.0, seed=0):
    """The tcgen05 forward on prepared fp16 operands -> (bf16 out (B, Hq, Sq, D), lse or None), plus the
    fp16 pre-scale output o16 when need_o16 (then the return is (out, lse, o16), all at the kernel's D).
    dropout_p > 0 drops softmax weights by the mask `seed` selects. Head dim 256 with few query blocks for
    the GPU runs the key-split schedule in a workspace from torch's allocator (tbf16_attn_fwd_ws)."""
    B, Hq, Sq, D = q16.shape
    Hkv, Sk = k16.shape[1], k16.shape[2]
    d_orig = d_orig or D
    sc = (1.0 / math.sqrt(d_orig)) if scale is None else float(scale)
    Dk = 64 if D <= 64 else 128 if D <= 128 else 256
    if D > 256:
        raise NotImplementedError("tbf16 attention on B200: head dims up to 256")
    if D != Dk:  # zero columns leave the logits unchanged and give zero output columns
        pad = (0, Dk - D)
        q16, k16, v16 = (torch.nn.functional.pad(t, pad) for t in (q16, k16, v16))
    dev = q16.device
    if need_o16 or Dk != D:
        out = torch.empty((B, Hq, Sq, Dk), device=dev, dtype=torch.bfloat16)
    else:  # (B, Sq, Hq, D) in memory, as torch's own SDPA returns it: the model's transpose + reshape to
        # (B, Sq, Hq D) rows for the output projection is then a view
        out = torch.empty((B, Sq, Hq, Dk), device=dev, dtype=torch.bfloat16).transpose(1, 2)
    lse_ld = (Sq + 127) // 128 * 128  # row stride the backward's bulk copies need
    lse = torch.empty((B, Hq, lse_ld), device=dev, dtype=torch.float32) if need_lse else None
    o16 = torch.empty((B, Hq, Sq, Dk), device=dev, dtype=torch.float16) if need_o16 else None
    m = additive_mask(attn_mask, B, Hq, Sq, Sk, dev)
    ms = m.stride()[:3] if m is not None else (0, 0, 0)
    args = (ptr(q16), ptr(k16), ptr(v16), B, Hq, Hkv, Sq, Sk, Dk, sc, int(bool(is_causal)), ptr(ev.contiguous()), ptr(m),
            *ms, ptr(out), *out.stride()[:3], ptr(lse), lse_ld, ptr(o16))
    ws_bytes = _fwd_ws_size(B, Hq, Hkv, Sq, Sk, Dk, bool(is_causal))
    ws = torch.empty(ws_bytes, device=dev, dtype=torch.uint8) if ws_bytes else None
    call("tbf16_attn_fwd_ws", *args, float(dropout_p), int(seed) if dropout_p else 0, ptr(ws), ws_bytes,
         stream_ptr(dev))
    if need_o16:
        return out, lse, o16
    if Dk != D:
        out = out[..., :D].contiguous()
    return out, lse


@torch.autocast("cuda", enabled=False)
def sdpa(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False):
    """Inference scaled attention (reference attention.py:56-65): V's max near 2^13 keeps channels far
    below it out of fp16's subnormals; the output is a convex combination of V rows, so it cannot
    overflow. dropout_p is applied as the reference passes it on to torch's SDPA (a fresh mask per call)."""
    if q.shape[1] != k.shape[1] and not enable_gqa:
        raise RuntimeError("tbf16.sdpa: different numbers of query and key heads need enable_gqa=True")
    D0 = q.shape[-1]
    q16, k16, v16, _, ev = prepare_qkv(q, k, v, v_exp=13)
    seed = dropout_seed() if dropout_p else 0
    out, _ = attn_forward(q16, k16, v16, ev, attn_mask, is_causal, scale, d_orig=D0, dropout_p=dropout_p, seed=seed)
    return out[..., :D0] if out.shape[-1] != D0 else out
