"""Multi-GPU partitions of the scaled path: one process per GPU, torch.distributed (NCCL over
NVLink/NVSwitch) for the one exchange that exists.

The path shards without changing any result:
  - linear over rows (M): row scales depend only on their own row, so each rank runs its rows against
    a replicated weight; nothing is exchanged (linear_rows).
  - linear column-parallel over N: each rank holds N/P weight rows with their scales and bias and
    computes y[:, its columns]; all_gather_into_tensor reassembles y (linear_column_parallel).
  - attention over batch x heads: each rank takes a slice of the heads. The reference takes eq and ek,
    the exponents that place q and k, as maxima over ALL (b, h) (attention.py:41), so the sharded call
    makes them global with one all_reduce(MAX) of two int32 and then scales exactly as the unsharded
    call would (prepare_qkv_sharded, sdpa_heads).
  - training attention over heads: the backward's dO exponent e = max_{b,h}(head_exp(dO) + ev_q) is
    also a global maximum (autograd.py:175), exchanged with one more all_reduce(MAX) of one int32
    before the backward kernel runs (global_dout_exponent, sdpa_heads_train).
The compute ops are parameters so the exchange logic can be checked on CPU with gloo.
"""
import math

import torch
import torch.distributed as dist

from . import attention, autograd
from ._ext import call, ptr, stream_ptr
from .ops import scaled_linear


def shard_range(n: int, rank: int, world: int, multiple: int = 1):
    """Contiguous [start, stop) of n items for `rank`, in blocks of `multiple` (balanced)."""
    blocks = (n + multiple - 1) // multiple
    per, extra = divmod(blocks, world)
    start = rank * per + min(rank, extra)
    stop = start + per + (1 if rank < extra else 0)
    return min(start * multiple, n), min(stop * multiple, n)


def linear_rows(x, w16, w_sinv, bias=None, linear=scaled_linear):
    """Row-sharded linear: this rank's rows of x against the full (replicated) weight. No collective."""
    return linear(x, w16, w_sinv, bias)


def shard_weight(w16, w_sinv, bias, rank, world):
    """This rank's column-parallel slice of a prepared weight (rows of w16 in multiples of 8)."""
    a, b = shard_range(w16.shape[0], rank, world, multiple=8)
    return w16[a:b].contiguous(), w_sinv[a:b].contiguous(), None if bias is None else bias[a:b].contiguous()


def linear_column_parallel(x, w16_shard, ws_shard, bias_shard=None, group=None, linear=scaled_linear):
    """y = x @ W^T with W's rows split across ranks: local y[:, shard], then all_gather over the group.
    Every rank's shard must have the same width (use shard_weight with N divisible by 8 * world)."""
    world = dist.get_world_size(group)
    y_local = linear(x, w16_shard, ws_shard, bias_shard)
    x_shape = y_local.shape[:-1]
    y2 = y_local.reshape(-1, y_local.shape[-1]).contiguous()
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty((world, *y2.shape), device=y2.device, dtype=y2.dtype)
        dist.all_gather_into_tensor(gathered, y2, group=group)
    else:  # gloo (CPU tests): no all_gather_into_tensor and no bf16; a gather is a copy, so move the bytes
        raw = torch.empty((world, y2.shape[0], y2.shape[1] * 2), device=y2.device, dtype=torch.uint8)
        dist.all_gather(list(raw.unbind(0)), y2.view(torch.uint8), group=group)
        gathered = raw.view(y2.dtype)
    return gathered.permute(1, 0, 2).reshape(*x_shape, world * y2.shape[-1])


def global_qk_exponents(q, k, group=None, head_exp=attention.head_exp):
    """(eq, ek): maxima over every rank's (b, h) of the q and k head exponents (attention.py:41)."""
    e = torch.stack([head_exp(q).amax(), head_exp(k).amax()]).to(torch.int32)
    dist.all_reduce(e, op=dist.ReduceOp.MAX, group=group)
    return e[0], e[1]


def _prepare_qkv_sharded_device(q, k, v, v_exp, group):
    """The CUDA form of prepare_qkv_sharded: tbf16_qkv_local_exponents (this rank's eq, ek and the head
    maxima), one all_reduce(MAX) of the two int32, tbf16_prepare_qkv_global (a, ev and the fp16 copies):
    two C calls and one collective, no host synchronisation."""
    D0 = q.shape[-1]
    q, k, v = (attention._as_kernel_layout(t) for t in (q, k, v))
    if not (q.dtype == k.dtype == v.dtype == torch.bfloat16):
        raise RuntimeError("tbf16.prepare_qkv_sharded: bf16 q, k, v expected")
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    if k.shape[0] != B or k.shape[3] != D or v.shape != k.shape or Hq % Hkv:
        raise RuntimeError(f"tbf16.prepare_qkv_sharded: incompatible shapes {tuple(q.shape)} {tuple(k.shape)}")
    dev = q.device
    eqk = torch.empty(2, device=dev, dtype=torch.int32)
    ws = torch.empty(B * Hq + 2 * B * Hkv, device=dev, dtype=torch.float32)
    strides = (ptr(q), *q.stride()[:3], ptr(k), *k.stride()[:3], ptr(v), *v.stride()[:3], B, Hq, Hkv, Sq, Sk, D)
    call("tbf16_qkv_local_exponents", *strides, ptr(eqk), ptr(ws), stream_ptr(dev))
    dist.all_reduce(eqk, op=dist.ReduceOp.MAX, group=group)
    q16 = torch.empty((B, Hq, Sq, D), device=dev, dtype=torch.float16)
    k16 = torch.empty((B, Hkv, Sk, D), device=dev, dtype=torch.float16)
    v16 = torch.empty((B, Hkv, Sk, D), device=dev, dtype=torch.float16)
    a = torch.empty((), device=dev, dtype=torch.int32)
    ev = torch.empty((B, Hkv), device=dev, dtype=torch.int32)
    call("tbf16_prepare_qkv_global", *strides, int(v_exp), ptr(eqk), ptr(ws), ptr(q16), ptr(k16), ptr(v16), ptr(a),
         ptr(ev), stream_ptr(dev))
    if D != D0:  # the kernels' 8-element padding, sliced back as head_scale does
        q16, k16, v16 = (t[..., :D0].contiguous() for t in (q16, k16, v16))
    return q16, k16, v16, a, ev


def prepare_qkv_sharded(q, k, v, v_exp=0, group=None, head_exp=attention.head_exp, head_scale=attention.head_scale):
    """prepare_qkv for this rank's heads with the global eq, ek: (q16, k16, v16, a, ev), identical to the
    corresponding slice of the unsharded prepare_qkv (ev is per (b, h_kv), so it needs no exchange).
    On CUDA with the library's own ops this is two C calls around one all_reduce; with other head_exp /
    head_scale (the CPU checks of the exchange over gloo) it is composed from them."""
    if q.is_cuda and head_exp is attention.head_exp and head_scale is attention.head_scale:
        return _prepare_qkv_sharded_device(q, k, v, v_exp, group)
    eq, ek = global_qk_exponents(q, k, group, head_exp)
    a = torch.div(ek - eq, 2, rounding_mode="floor")
    a = torch.maximum(torch.minimum(a, 14 - eq), ek - 14)
    ev = head_exp(v) - v_exp
    return head_scale(q, a, torch.float16), head_scale(k, -a, torch.float16), head_scale(v, -ev, torch.float16), a, ev


@torch.autocast("cuda", enabled=False)
def sdpa_heads(q, k, v, attn_mask=None, is_causal=False, scale=None, enable_gqa=False, group=None):
    """Inference scaled attention on this rank's heads (q, k, v already sliced by head; GQA groups must not
    straddle ranks). Same result as the matching heads of tbf16.sdpa on the full tensors."""
    D0 = q.shape[-1]
    q16, k16, v16, _, ev = prepare_qkv_sharded(q, k, v, v_exp=13, group=group)
    out, _ = attention.attn_forward(q16, k16, v16, ev, attn_mask, is_causal, scale, d_orig=D0)
    return out[..., :D0] if out.shape[-1] != D0 else out


def global_dout_exponent(dout, ev, group=None, head_exp=attention.head_exp):
    """(e_local, e_global) as int32 tensors: max over this rank's (b, h) and over every rank's of
    head_exp(dout) + ev_q, the exponent that fixes the backward's dO scale 2^G, G = t_do - e
    (reference autograd.py:173-178). ev: this rank's per-(b, h_kv) V exponents."""
    ev_q = attention.expand_heads(ev, dout.shape[1])
    e_local = (head_exp(dout) + ev_q).amax().to(torch.int32).reshape(1)
    e_global = e_local.clone()
    dist.all_reduce(e_global, op=dist.ReduceOp.MAX, group=group)
    return e_local[0], e_global[0]


class _ShardedSDPAFn(torch.autograd.Function):
    """Training attention on this rank's heads with the unsharded call's scales: the forward's a from the
    global eq, ek (prepare_qkv_sharded); the backward's G from the global dO exponent, which stays on the
    device (all_reduce into an int32 the backward kernel reads: tbf16_attn_bwd_sharded)."""

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def forward(ctx, q, k, v, attn_mask, is_causal, scale, group):
        D0 = q.shape[-1]
        if D0 > 256:
            raise NotImplementedError("tbf16 sharded training attention: head dims up to 256")
        q16, k16, v16, a, ev = prepare_qkv_sharded(q, k, v, v_exp=0, group=group)
        Dk = 64 if D0 <= 64 else 128 if D0 <= 128 else 256
        if Dk != D0:
            q16, k16, v16 = (torch.nn.functional.pad(t, (0, Dk - D0)) for t in (q16, k16, v16))
        sc = 1.0 / math.sqrt(D0) if scale is None else float(scale)
        B, Hq, Sq, _ = q16.shape
        mask16 = attention.additive_mask(attn_mask, B, Hq, Sq, k.shape[2], q.device)
        out, lse, o16 = attention.attn_forward(q16, k16, v16, ev, mask16, is_causal, sc, need_lse=True, need_o16=True)
        ctx.save_for_backward(q16, k16, v16, o16, lse, a, ev, mask16)
        ctx.args = (is_causal, sc, D0, group)
        return out[..., :D0].contiguous() if Dk != D0 else out

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def backward(ctx, dout):
        q16, k16, v16, o16, lse, a, ev, mask16 = ctx.saved_tensors
        is_causal, sc, D0, group = ctx.args
        if D0 % 8:
            dout = torch.nn.functional.pad(dout, (0, 8 - D0 % 8))
        _, e_global = global_dout_exponent(dout, ev, group)
        dq, dk, dv, _ = autograd.attn_backward(q16, k16, v16, o16, lse, a, ev, dout, mask16, is_causal, sc, D0,
                                               e_global=e_global.reshape(1))
        if q16.shape[-1] != D0:
            dq, dk, dv = (t[..., :D0].contiguous() for t in (dq, dk, dv))
        return dq, dk, dv, None, None, None, None


def sdpa_heads_train(q, k, v, attn_mask=None, is_causal=False, scale=None, group=None):
    """Differentiable scaled attention on this rank's heads (q, k, v sliced by head, GQA groups whole on
    one rank): forward and gradients equal the matching heads of tbf16.autograd.sdpa on the full tensors."""
    return _ShardedSDPAFn.apply(q, k, v, attn_mask, is_causal, scale, group)
