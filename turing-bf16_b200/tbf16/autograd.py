"""Differentiable scaled ops for training on the B200 kernels.

Public names as in the reference's tbf16/autograd.py: quantize_cols, ScaledLinearFn, FP32LinearFn,
linear, ScaledSDPAFn, sdpa, CHECK_OVERFLOW.

Linear backward: dX = dY W contracts over N and dW = dY^T X over M, so the operands whose contraction
axis changed are given power-of-two scales per column instead of per row (the reference's exponent
conventions for each operand, autograd.py:71-90 there). The three products run on the tcgen05 GEMM,
which reads the column-scaled operands MN-major from their row-major storage and writes bf16 from
its fp32 accumulator.

Attention: the tcgen05 flash-attention forward and backward. The backward multiplies dO by 2^G, G
chosen per call from the head exponents so that dS stays inside fp16's normal range; a kernel that
still meets a non-finite value raises a device flag and the call is repeated with G lowered by 8, at
most six times (the reference's retry, autograd.py:177-189). Gradients leave the kernel from fp32
accumulators, so the retry is a safety net rather than a regular path.
"""
import math
import os

import torch
import torch.nn.functional as F

from . import attention, ops
from ._ext import call, lib, ptr, require_cuda, stream_ptr

# Whether the attention backward reads the kernel's non-finite flag (one host synchronisation per call) and
# retries at a smaller dO scale; TBF16_ATTN_CHECK=0 skips the read and the retry.
CHECK_OVERFLOW = os.environ.get("TBF16_ATTN_CHECK", "1") != "0"


def quantize_cols(x: torch.Tensor, target_exp: int = 0, row_mul=None):
    """bf16 (R, K) -> (fp16 (R, K), fp32 (K,) inverse scales), one power-of-two scale per column.
    row_mul (R,) powers of two, optional: quantize x * row_mul[:, None] instead (exact)."""
    require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise RuntimeError("tbf16.quantize_cols: 2-D bf16 CUDA tensor expected")
    if x.stride(1) != 1 or x.shape[1] % 8 or (x.shape[0] > 1 and x.stride(0) % 8) or x.data_ptr() % 16:
        x = ops._pad_cols(x)
    R, K = x.shape
    y = torch.empty((R, K), device=x.device, dtype=torch.float16)
    s_inv = torch.empty((K,), device=x.device, dtype=torch.float32)
    ws = torch.empty((K,), device=x.device, dtype=torch.float32)
    rm = None if row_mul is None else row_mul.contiguous().float()
    call("tbf16_quantize_cols", ptr(x), R, K, x.stride(0) if R > 1 else K, int(target_exp), ptr(rm), ptr(y), K,
         ptr(s_inv), ptr(ws), stream_ptr(x.device))
    return y, s_inv


@torch.autocast("cuda", enabled=False)
def _scaled_mm(a16, sa, b16, sb, a_mn=False, b_mn=False):
    """(A @ B^T) * sa[:, None] * sb[None, :] as bf16, with A = a16 (M, K) or a16 (K, M) if a_mn, and
    B = b16 (N, K) or b16 (K, N) if b_mn (reference autograd.py:114-120 took a16 @ b16 explicitly)."""
    M = a16.shape[1] if a_mn else a16.shape[0]
    K = a16.shape[0] if a_mn else a16.shape[1]
    N = b16.shape[1] if b_mn else b16.shape[0]
    return ops._gemm_f16(a16, a_mn, b16, b_mn, M, N, K, sa, sb)


def _aligned(*ts):
    return all(t.shape[-1] % 8 == 0 and t.stride(-1) == 1 and t.data_ptr() % 16 == 0 for t in ts)


class ScaledLinearFn(torch.autograd.Function):
    """y = x W^T + b for bf16 x and W. What the backward needs is kept in the forward's own form: x's
    fp16 rows and inverse row scales (as many bytes as x; dW folds the scales into dY's columns) and W,
    which the backward scales by columns."""

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def forward(ctx, x, w, bias):
        rows16, rows_sinv = ops.quantize_rows_shared(x)  # one fp16 copy for sibling layers reading x
        y = ops.linear_q(rows16, rows_sinv, *ops.prepare_weight(w), bias)
        ctx.save_for_backward(rows16, rows_sinv, w)
        ctx.x_shape, ctx.has_bias = x.shape, bias is not None
        return y.reshape(*x.shape[:-1], w.shape[0])

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def backward(ctx, dy):
        x16, sx, w = ctx.saved_tensors
        return _linear_backward(dy, x16, sx, w, ctx.needs_input_grad[0], ctx.needs_input_grad[1],
                                ctx.has_bias and ctx.needs_input_grad[2], ctx.x_shape)


def _linear_backward(dy, x16, sx, w, want_dx, want_dw, want_db, x_shape):
    """dX, dW, db of y = x W^T + b from the forward's fp16 rows x16 and inverse row scales sx."""
    N, K = w.shape
    dy2 = dy.reshape(-1, N).contiguous()
    if dy2.dtype != torch.bfloat16:
        dy2 = dy2.bfloat16()
    M = dy2.shape[0]
    dx = dw = db = None
    pad = N % 8 or K % 8
    if want_dx:  # contraction over N: dY rows (L1, t=15) x W columns (t = _target_exp(N))
        t = ops._target_exp(N)
        dy16, sdy = ops.quantize_rows(dy2, ops.L1_TARGET, l1=True)
        w16c, swc = quantize_cols(w.contiguous(), t)
        if pad:
            dx = _padded_mm(dy16, sdy, w16c, swc, M, N, K, kind="dx")
        else:
            dx = _scaled_mm(dy16, sdy, w16c, swc, a_mn=False, b_mn=True)  # B[k, n] = w16c[n, k]
        dx = dx.reshape(x_shape)
    if want_dw:  # contraction over M: dW[n, k] = sum_m dy[m, n] sx[m] x16[m, k]
        # |x16| < 1, so |dW16| < M * 2^t; keep that under fp16's max (reference autograd.py:84-87).
        t = min(0, 15 - math.ceil(math.log2(max(M, 1))))
        dy16c, sdyc = quantize_cols(dy2, t, sx.reshape(-1))
        x16 = x16.reshape(M, K)
        if pad:
            dw = _padded_mm(dy16c, sdyc, x16, None, M, N, K, kind="dw")
        else:
            dw = _scaled_mm(dy16c, sdyc, x16, None, a_mn=True, b_mn=True)
    if want_db:
        db = dy2.float().sum(0).to(dy.dtype)
    return dx, dw, db


class GLULinearFn(torch.autograd.Function):
    """y = (act(gate) * up) W^T + b for training, with the gated activation fused: forward, the
    producer-fused rows (tbf16_glu_rows: h's fp16 operand and row scales in one pass, no row pass in the
    linear); backward, the linear's dX and dW as ScaledLinearFn's (h's fp16 rows stand in for x16) and
    d_gate, d_up in one pass (tbf16_glu_bwd, torch's autograd arithmetic for act(g) * u on bf16).
    Needs I (gate's last dimension) a multiple of 8."""

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def forward(ctx, gate, up, w, bias, act):
        N, I = w.shape
        h16, s_inv = ops.glu_rows(gate, up, act)
        w16, sw = ops.prepare_weight(w)
        ctx.save_for_backward(gate, up, h16, s_inv, w)
        ctx.act, ctx.has_bias = act, bias is not None
        return ops.linear_q(h16.reshape(-1, I), s_inv.reshape(-1), w16, sw, bias).reshape(*gate.shape[:-1], N)

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def backward(ctx, dy):
        gate, up, h16, s_inv, w = ctx.saved_tensors
        want_gu = ctx.needs_input_grad[0] or ctx.needs_input_grad[1]
        dh, dw, db = _linear_backward(dy, h16, s_inv, w, want_gu, ctx.needs_input_grad[2],
                                      ctx.has_bias and ctx.needs_input_grad[3], gate.shape)
        dg = du = None
        if want_gu:
            dg, du = ops.glu_bwd(dh.to(torch.bfloat16), gate, up, ctx.act)
        return dg, du, dw, db, None


def glu_linear(gate, up, w, bias=None, act="silu"):
    """Training form of linear(act(gate) * up, w, bias) with the activation fused into the linear's
    input pass and its backward (GLULinearFn); act: "silu" or "gelu_tanh". Falls back to the unfused
    composition for inputs the fused kernels do not take (row length not a multiple of 8 or above
    16384, non-bf16)."""
    I = gate.shape[-1]
    if (gate.dtype == up.dtype == torch.bfloat16 and I % 8 == 0 and I <= 16384 and w.shape[1] == I
            and gate.is_cuda):
        return GLULinearFn.apply(gate, up, w, bias, act)
    a = F.silu(gate) if act == "silu" else F.gelu(gate, approximate="tanh")
    return linear(a * up, w, bias)


def _padded_mm(a16, sa, b16, sb, M, N, K, kind):
    """dX / dW for layers whose N or K is not a multiple of 8: zero-pad the fp16 operands so every
    row is 16-byte aligned, run the same GEMM, slice the result."""
    Np, Kp = (N + 7) // 8 * 8, (K + 7) // 8 * 8
    dev = a16.device
    if kind == "dx":  # a16 = dy16 (M, Np'), b16 = w16c (N, K') -> dX (M, K)
        A = torch.zeros(M, Np, device=dev, dtype=torch.float16)
        A[:, :N] = a16[:, :N]
        Bm = torch.zeros(Np, Kp, device=dev, dtype=torch.float16)
        Bm[:N, :K] = b16[:N, :K]
        sbp = torch.ones(Kp, device=dev)
        sbp[:K] = sb[:K]
        return ops._gemm_f16(A, 0, Bm, 1, M, Kp, Np, sa, sbp)[:, :K]
    # dw: a16 = dy16c (M, N'), b16 = x16 (M, K') -> dW (N, K)
    A = torch.zeros(M, Np, device=dev, dtype=torch.float16)
    A[:, :N] = a16[:, :N]
    Bm = torch.zeros(M, Kp, device=dev, dtype=torch.float16)
    Bm[:, :K] = b16[:, :K]
    sap = torch.ones(Np, device=dev)
    sap[:N] = sa[:N]
    return ops._gemm_f16(A, 1, Bm, 1, Np, Kp, M, sap, None)[:N, :K]


class FP32LinearFn(torch.autograd.Function):
    """Layers with a dimension below convert.MIN_DIM (LoRA adapters and the like; the reference's
    autograd.py:93-112 role): fp32 GEMMs over the bf16 tensors with bf16 results. The saved x is the
    caller's bf16 tensor itself, so adapters that read the same input share it."""

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def forward(ctx, x, w, bias):
        ctx.save_for_backward(x, w)
        ctx.with_bias = bias is not None
        y = torch.matmul(x.float(), w.float().t())
        return (y if bias is None else y + bias.float()).to(x.dtype)

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        need_x, need_w, need_b = ctx.needs_input_grad
        g = dy.float().reshape(-1, w.shape[0])
        dx = (g @ w.float()).reshape(x.shape).to(x.dtype) if need_x else None
        dw = (g.t() @ x.reshape(-1, w.shape[1]).float()).to(w.dtype) if need_w else None
        db = g.sum(0).to(dy.dtype) if need_b and ctx.with_bias else None
        return dx, dw, db


def linear(x, w, bias=None):
    """F.linear(x, w, bias) with gradients, for bf16 x and w, on the scaled kernels (ScaledLinearFn)."""
    return ScaledLinearFn.apply(x, w, bias)


def attn_backward(q16, k16, v16, o16, lse, a, ev, dout, mask16, is_causal, scale, d_orig, t_do_offset=0,
                  dropout_p=0.0, seed=0, e_global=None):
    """Runs tbf16_attn_bwd with the reference's retry loop: t_do = 12 - ceil(log2 d), lowered by 8 and
    redone while the kernel reports a non-finite value (at most 6 attempts). t_do_offset (>= 0) lowers
    the target further: a head-sharded call passes how far the global dO exponent exceeds its own heads'
    maximum, so G comes out as the unsharded call's; or, without a host round trip, e_global: a device
    int32 holding that global exponent (tbf16_attn_bwd_sharded). dropout_p, seed: the forward's mask."""
    B, Hq, Sq, Dk = q16.shape
    Hkv, Sk = k16.shape[1], k16.shape[2]
    dev = q16.device
    if dout.dtype != torch.bfloat16:
        dout = dout.bfloat16()
    if not attention._fast(dout):
        dout = dout.contiguous()
    dq = torch.empty((B, Hq, Sq, Dk), device=dev, dtype=torch.bfloat16)
    dk = torch.empty((B, Hkv, Sk, Dk), device=dev, dtype=torch.bfloat16)
    dv = torch.empty((B, Hkv, Sk, Dk), device=dev, dtype=torch.bfloat16)
    G = torch.empty((), device=dev, dtype=torch.int32)
    flag = torch.zeros((), device=dev, dtype=torch.int32)
    nbytes = lib().tbf16_attn_bwd_workspace_size(B, Hq, Hkv, Sq, Sk, Dk)
    ws = torch.empty(nbytes, device=dev, dtype=torch.uint8)
    ms = mask16.stride()[:3] if mask16 is not None else (0, 0, 0)
    t_do = 12 - math.ceil(math.log2(d_orig)) - int(t_do_offset)
    for _attempt in range(6):
        flag.zero_()
        args = (ptr(q16), ptr(k16), ptr(v16), ptr(o16), ptr(lse), lse.shape[-1], ptr(dout), *dout.stride()[:3],
                dout.shape[-1], ptr(a), ptr(ev), B, Hq, Hkv, Sq, Sk, Dk, float(scale), int(bool(is_causal)), ptr(mask16),
                *ms, int(t_do), ptr(dq), ptr(dk), ptr(dv), ptr(G), ptr(flag), ptr(ws), nbytes)
        if e_global is not None:
            call("tbf16_attn_bwd_sharded", *args, float(dropout_p), int(seed), ptr(e_global), stream_ptr(dev))
        elif dropout_p:
            call("tbf16_attn_bwd_dropout", *args, float(dropout_p), int(seed), stream_ptr(dev))
        else:
            call("tbf16_attn_bwd", *args, stream_ptr(dev))
        if not CHECK_OVERFLOW:
            break
        if not bool(flag):  # host sync, once per attention call
            break
        t_do -= 8
    else:
        raise FloatingPointError("tbf16 attention backward overflowed fp16 even after rescaling")
    return dq, dk, dv, G


class ScaledSDPAFn(torch.autograd.Function):
    """Scaled attention forward and backward on the tcgen05 kernels; keeps everything in
    save_for_backward, so activation checkpointing can drop and recompute it."""

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def forward(ctx, q, k, v, attn_mask, dropout_p, is_causal, scale, enable_gqa):
        if q.shape[1] != k.shape[1] and not enable_gqa:
            raise RuntimeError("tbf16.sdpa: different numbers of query and key heads need enable_gqa=True")
        D0 = q.shape[-1]
        q16, k16, v16, a, ev = attention.prepare_qkv(q, k, v)
        B, Hq, Sq, D = q16.shape
        if D > 256:
            raise NotImplementedError("tbf16 attention on B200: head dims up to 256")
        Dk = 64 if D <= 64 else 128 if D <= 128 else 256
        if Dk != D:
            q16, k16, v16 = (F.pad(t, (0, Dk - D)) for t in (q16, k16, v16))
        sc = 1.0 / math.sqrt(D0) if scale is None else float(scale)
        mask16 = attention.additive_mask(attn_mask, B, Hq, Sq, k.shape[2], q.device)
        seed = attention.dropout_seed() if dropout_p else 0
        out, lse, o16 = attention.attn_forward(q16, k16, v16, ev, mask16, is_causal, sc, need_lse=True, need_o16=True,
                                               dropout_p=dropout_p, seed=seed)
        ctx.save_for_backward(q16, k16, v16, o16, lse, a, ev, mask16)
        ctx.args = (is_causal, sc, D0, float(dropout_p), seed)
        return out[..., :D0].contiguous() if Dk != D0 else out

    @staticmethod
    @torch.autocast("cuda", enabled=False)
    def backward(ctx, dout):
        q16, k16, v16, o16, lse, a, ev, mask16 = ctx.saved_tensors
        is_causal, sc, D0, dropout_p, seed = ctx.args
        Dk = q16.shape[-1]
        if D0 % 8:
            dout = F.pad(dout, (0, 8 - D0 % 8))
        dq, dk, dv, _ = attn_backward(q16, k16, v16, o16, lse, a, ev, dout, mask16, is_causal, sc, D0,
                                      dropout_p=dropout_p, seed=seed)
        if Dk != D0:
            dq, dk, dv = (t[..., :D0].contiguous() for t in (dq, dk, dv))
        return dq, dk, dv, None, None, None, None, None


def sdpa(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None, enable_gqa=False):
    """Differentiable bf16 scaled_dot_product_attention on fp16 tensor cores."""
    return ScaledSDPAFn.apply(q, k, v, attn_mask, dropout_p, is_causal, scale, enable_gqa)
