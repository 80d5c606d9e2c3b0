"""CPU oracle for tbf16's hot path (TEST INFRASTRUCTURE ONLY).

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg; the tbf16 package
never imports it. Integer and rounding steps run in the C restatement (tbf16_oracle.c, through
ctypes); the attention and training algorithms are restated here in fp64 torch on CPU, on top of
those bit-exact fp16 operands. Each function cites the reference file:line it follows (paths
relative to the tech-cosmos/turing-bf16 project root).

Parity is pinned: tests/test_oracle_golden.py checks this module against vectors produced by the
reference's own code run on CPU (tests/golden/make_golden.py), and tests/test_oracle_kat.py
checks the exponent rules on known answers derived from the cited CUDA lines.
"""
import ctypes
import math
import os
import pathlib
import subprocess

import numpy as np
import torch

_HERE = pathlib.Path(__file__).resolve().parent
_LIB = None

_i64, _i32, _f32p, _u16p = ctypes.c_int64, ctypes.c_int, ctypes.POINTER(ctypes.c_float), ctypes.c_void_p


def build():
    """Compile tbf16_oracle.c into oracle/_build/liboracle.so (gcc, seconds)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = _HERE / "_build" / "liboracle.so"
        if not path.exists() or path.stat().st_mtime < (_HERE / "tbf16_oracle.c").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(path))
        vp = ctypes.c_void_p
        sig = {
            "orc_pow2_scale_array": [vp, _i64, _i32, _i32, vp],
            "orc_frexp_exp_array": [vp, _i64, vp],
            "orc_row_reduce": [vp, _i64, _i64, _i64, _i32, vp],
            "orc_quantize_rows": [vp, _i64, _i64, _i64, _i32, _i32, vp, _i64, vp],
            "orc_row_scale_fused": [vp, _i64, _i64, _i64, _i32, _i32, vp],
            "orc_quantize_cols": [vp, _i64, _i64, _i64, _i32, vp, vp, _i64, vp],
            "orc_head_amax": [vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, vp],
            "orc_head_scale_cast": [vp, _i32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, vp, vp, _i32],
            "orc_linear_fused": [vp, _i64, _i64, _i64, vp, _i64, _i64, vp, vp, _i32, _i32, vp, _i64, vp],
            "orc_gemm_f16": [vp, _i32, _i64, vp, _i32, _i64, _i64, _i64, _i64, vp, vp, vp, vp, _i64],
            "orc_f32_to_f16_array": [vp, vp, _i64],
            "orc_f32_to_bf16_array": [vp, vp, _i64],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = None
        _LIB = L
    return _LIB


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _cpu(t):
    return t.detach().to("cpu")


# ----------------------------------------------------------------------------- exponent rules

def target_exp(K: int) -> int:
    """tbf16/ops.py:29-32: t = min(0, floor((15 - ceil(log2 K)) / 2))."""
    return min(0, (15 - math.ceil(math.log2(max(K, 1)))) // 2)


def pow2_scale(amax: torch.Tensor, t: int, kind: str = "small") -> torch.Tensor:
    """Power-of-two scales from exponent bits. kind 'small' = small_kernels.cu:12-18, 'fused' =
    gemm_sm75.cu:19-23, 'triton' = ops.py:39-45 (times 2^t)."""
    a = _cpu(amax).float().contiguous()
    out = torch.empty_like(a)
    lib().orc_pow2_scale_array(_p(a), a.numel(), t, {"small": 0, "fused": 1, "triton": 2}[kind], _p(out))
    return out


def frexp_exp(x: torch.Tensor) -> torch.Tensor:
    """Exponent of torch.frexp (attention.py:27) from the fp32 bits."""
    a = _cpu(x).float().contiguous()
    out = torch.empty(a.shape, dtype=torch.int32)
    lib().orc_frexp_exp_array(_p(a), a.numel(), _p(out))
    return out


def f16_rn(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> fp16, round to nearest even (IEEE restatement in C)."""
    a = _cpu(x).float().contiguous()
    out = torch.empty(a.shape, dtype=torch.float16)
    lib().orc_f32_to_f16_array(_p(a), _p(out), a.numel())
    return out


def bf16_rn(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16, round to nearest even. fp64 inputs are first rounded to fp32 (as a GPU
    epilogue does when it forms the fp32 value it converts)."""
    a = _cpu(x).float().contiguous()
    out = torch.empty(a.shape, dtype=torch.bfloat16)
    lib().orc_f32_to_bf16_array(_p(a), _p(out), a.numel())
    return out


# ----------------------------------------------------------------------------- row / column scales

def row_reduce(x: torch.Tensor, l1: bool = False) -> torch.Tensor:
    """Row max |x| (NaN ignored) or exact L1 norm rounded to fp32 (small_kernels.cu:42-60)."""
    x = _cpu(x)
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    out = torch.empty(x.shape[0], dtype=torch.float32)
    lib().orc_row_reduce(_p(x), x.shape[0], x.shape[1], x.stride(0), int(l1), _p(out))
    return out


def quantize_rows(x: torch.Tensor, target_exp: int = 0, l1: bool = False):
    """tbf16/ops.py:74-89 -> small_kernels.cu:35-74: (fp16 (R, K), fp32 (R,) inverse scales)."""
    x = _cpu(x)
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    R, K = x.shape
    y = torch.empty((R, K), dtype=torch.float16)
    s_inv = torch.empty(R, dtype=torch.float32)
    lib().orc_quantize_rows(_p(x), R, K, x.stride(0), target_exp, int(l1), _p(y), K, _p(s_inv))
    return y, s_inv


def row_scale_fused(x: torch.Tensor, target_exp: int = 15, l1: bool = False) -> torch.Tensor:
    """tbf16/csrc/gemm_sm75.cu:27-47,243-253: fp32 (M,) inverse row scales of the fused GEMM."""
    x = _cpu(x)
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    out = torch.empty(x.shape[0], dtype=torch.float32)
    lib().orc_row_scale_fused(_p(x), x.shape[0], x.shape[1], x.stride(0), target_exp, int(l1), _p(out))
    return out


def prepare_weight(w: torch.Tensor):
    """tbf16/ops.py:140-142: quantize_rows(w, _target_exp(K))."""
    return quantize_rows(_cpu(w).contiguous(), target_exp(w.shape[1]))


def quantize_cols(x: torch.Tensor, target_exp: int = 0, row_mul=None):
    """tbf16/autograd.py:26-36 -> small_kernels.cu:136-184,318-340: (fp16 (R, K), fp32 (K,))."""
    x = _cpu(x)
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    R, K = x.shape
    rm = None if row_mul is None else _cpu(row_mul).float().contiguous()
    y = torch.empty((R, K), dtype=torch.float16)
    s_inv = torch.empty(K, dtype=torch.float32)
    lib().orc_quantize_cols(_p(x), R, K, x.stride(0), target_exp, _p(rm), _p(y), K, _p(s_inv))
    return y, s_inv


# ----------------------------------------------------------------------------- attention helpers

def head_amax(x: torch.Tensor) -> torch.Tensor:
    """small_kernels.cu:221-243,342-359: fp32 (B, H) amax of a strided (B, H, S, D) tensor."""
    x = _cpu(x)
    assert x.dim() == 4 and x.stride(3) == 1 and x.dtype in (torch.bfloat16, torch.float16)
    B, H, S, D = x.shape
    out = torch.empty((B, H), dtype=torch.float32)
    lib().orc_head_amax(_p(x), int(x.dtype == torch.float16), B, H, S, D, x.stride(0), x.stride(1), x.stride(2),
                        _p(out))
    return out


def head_exp(x: torch.Tensor) -> torch.Tensor:
    """tbf16/attention.py:24-27: int32 (B, H) frexp exponent of each head's amax."""
    return frexp_exp(head_amax(x))


def head_scale(x: torch.Tensor, e: torch.Tensor, dtype) -> torch.Tensor:
    """tbf16/attention.py:30-35 -> small_kernels.cu:246-263: contiguous cast(x * 2^e[b, h])."""
    x = _cpu(x)
    if x.stride(-1) != 1:
        x = x.contiguous()
    B, H, S, D = x.shape
    e = _cpu(e).to(torch.int32).expand(B, H).contiguous()
    y = torch.empty((B, H, S, D), dtype=dtype)
    lib().orc_head_scale_cast(_p(x), int(x.dtype == torch.float16), B, H, S, D, x.stride(0), x.stride(1),
                              x.stride(2), _p(e), _p(y), int(dtype == torch.float16))
    return y


def expand_heads(e: torch.Tensor, n_heads: int) -> torch.Tensor:
    """tbf16/attention.py:51-53."""
    return e if e.shape[1] == n_heads else e.repeat_interleave(n_heads // e.shape[1], dim=1)


def prepare_exponents(q, k, v, v_exp=0):
    """tbf16/attention.py:41-46: a = clamp(floor((ek - eq) / 2), ek - 14, 14 - eq) with eq, ek the
    maxima over all (b, h); ev = head_exp(v) - v_exp per (b, h_kv). Returns int32 tensors."""
    eq, ek = head_exp(q).max(), head_exp(k).max()
    a = torch.div(ek - eq, 2, rounding_mode="floor")
    a = torch.maximum(torch.minimum(a, 14 - eq), ek - 14)
    ev = head_exp(v) - v_exp
    return a.to(torch.int32), ev.to(torch.int32)


def prepare_qkv(q, k, v, v_exp=0):
    """tbf16/attention.py:38-48: (q16, k16, v16, a, ev)."""
    a, ev = prepare_exponents(q, k, v, v_exp)
    return (head_scale(q, a, torch.float16), head_scale(k, -a, torch.float16), head_scale(v, -ev, torch.float16),
            a, ev)


def _expand_kv(t, n_heads):
    return t if t.shape[1] == n_heads else t.repeat_interleave(n_heads // t.shape[1], dim=1)


def _logit_mask(attn_mask, is_causal, Sq, Sk):
    """Additive fp64 mask: bool -> 0 / -inf; float masks are cast to fp16 first as the reference
    does (attention.py:61-62, autograd.py:124-134); is_causal keeps key j <= query i (top-left)."""
    m = None
    if attn_mask is not None:
        am = _cpu(attn_mask)
        if am.dtype == torch.bool:
            m = torch.zeros(am.shape, dtype=torch.float64).masked_fill_(~am, float("-inf"))
        else:
            m = am.to(torch.float16).double()
    if is_causal:
        c = torch.ones(Sq, Sk, dtype=torch.bool).tril()
        cm = torch.zeros(Sq, Sk, dtype=torch.float64).masked_fill_(~c, float("-inf"))
        m = cm if m is None else m + cm
    return m


def _select_kv_heads(t, kv_heads, group):
    """Stacks the (b, hkv) head groups of t (B, H, S, D) along a new batch axis: query tensors give
    (n, group, S, D), key / value tensors (group = 1) give (n, 1, S, D)."""
    return torch.stack([t[b, h * group:(h + 1) * group] for b, h in kv_heads])


def _select_mask(m, kv_heads, group):
    if m is None or m.dim() < 4:
        return m
    return torch.stack([m[b if m.shape[0] > 1 else 0, h * group:(h + 1) * group] if m.shape[1] > 1
                        else m[b if m.shape[0] > 1 else 0] for b, h in kv_heads])


def sdpa_fwd(q, k, v, attn_mask=None, is_causal=False, scale=None, v_exp=13, kv_heads=None):
    """Scaled attention forward, tbf16/attention.py:56-65 (v_exp=13, inference) and
    tbf16/autograd.py:153-164 (v_exp=0, training), computed in fp64 from the exact fp16 copies.

    Returns a dict: out (bf16 of O * 2^ev rounded once, this build's epilogue), out_ref (the
    reference's fp16 out16 rounded again to bf16 by head_scale, attention.py:65), lse (natural-log
    logsumexp of the scaled logits, fp64), o16 (fp64 O before the 2^ev rescale), p, and the
    integer exponents a, ev.

    kv_heads: optional list of (b, h_kv) pairs. The exponents a and ev are still taken over every
    head (they are global maxima in the reference), but the fp64 attention is computed only for
    those KV heads and their query heads, stacked along the batch axis: every returned tensor then
    has shape (len(kv_heads), group, ...) for query-side values and (len(kv_heads), 1, ...) for ev."""
    q16, k16, v16, a, ev = prepare_qkv(q, k, v, v_exp)
    B, Hq, Sq, D = q16.shape
    Sk = k16.shape[2]
    sc = scale if scale is not None else 1.0 / math.sqrt(D)
    m = _logit_mask(attn_mask, is_causal, Sq, Sk)
    if kv_heads is not None:
        group = Hq // k16.shape[1]
        q16, k16, v16 = (_select_kv_heads(q16, kv_heads, group), _select_kv_heads(k16, kv_heads, 1),
                         _select_kv_heads(v16, kv_heads, 1))
        ev = torch.stack([ev[b, h:h + 1] for b, h in kv_heads])
        m = _select_mask(m, kv_heads, group)
        Hq = group
    kk, vv = _expand_kv(k16, Hq).double(), _expand_kv(v16, Hq).double()
    s = (q16.double() @ kk.transpose(-1, -2)) * sc
    if m is not None:
        s = s + m
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse[..., None])
    o = p @ vv
    zmax = torch.where(torch.isfinite(s), s.abs(), torch.zeros_like(s)).amax(-1)  # largest |scaled logit| per row
    ev_q = expand_heads(ev, Hq)
    scale_o = torch.ldexp(torch.ones(()), ev_q.double())[..., None, None]
    out = bf16_rn(o * scale_o)
    out_ref = bf16_rn(f16_rn(o).double() * scale_o)
    return {"out": out, "out_ref": out_ref, "lse": lse, "o16": o, "p": p, "a": a, "ev": ev, "q16": q16,
            "k16": k16, "v16": v16, "scale": sc, "zmax": zmax, "pv_abs": p @ vv.abs()}


def sdpa_bwd(q, k, v, dout, attn_mask=None, is_causal=False, scale=None, kv_heads=None):
    """Scaled attention backward, tbf16/autograd.py:166-193, in fp64 from the exact fp16 operands:
    G = (12 - ceil(log2 D)) - max_{b,h}(head_exp(dout) + ev_q); dO16 = fp16(dout * 2^(ev_q + G));
    dq = dq16 * 2^(a - G), dk = reduce_kv(dk16) * 2^(-a - G), dv = reduce_kv(dv16) * 2^(-ev - G),
    each rounded once to bf16 (the reference rounds dq16/dk16/dv16 to fp16 first). The retry loop
    (:177-189) never triggers here because nothing is rounded to fp16 after dO16.

    Also returned for error bounds: abs_dq, abs_dk (the dQ / dK contractions over P (|dP| + sum |dO16| |O|),
    the magnitudes that the relative rounding of P, delta and dS scale with, scaled like the gradients),
    abs_dv (over P |dO16|), sub_dq / sub_dk / sub_dv (the same contractions with P replaced by 1: what the
    absolute 2^-25 rounding of fp16 values near zero scales with), and dq16 / dk16 / dv16 before their
    power-of-two scales (the reference rounds these to fp16). kv_heads: as in sdpa_fwd (G stays global)."""
    f = sdpa_fwd(q, k, v, attn_mask, is_causal, scale, v_exp=0, kv_heads=kv_heads)
    q16, k16, v16, a, ev, p, o = f["q16"], f["k16"], f["v16"], f["a"], f["ev"], f["p"], f["o16"]
    Hq = q16.shape[1]
    B_all, Hq_all = q.shape[0], q.shape[1]
    ev_full = prepare_exponents(q, k, v, 0)[1]
    e = (head_exp(dout) + expand_heads(ev_full, Hq_all)).max()
    D = q16.shape[-1]
    t_do = 12 - math.ceil(math.log2(D))
    G = int(t_do - e)
    if kv_heads is not None:
        dout = _select_kv_heads(_cpu(dout), kv_heads, Hq_all // k.shape[1])
    B = q16.shape[0]
    Hkv = k16.shape[1]
    ev_q = expand_heads(ev, Hq)
    do16 = head_scale(dout, ev_q + G, torch.float16).double()
    kk, vv = _expand_kv(k16, Hq).double(), _expand_kv(v16, Hq).double()
    dv16 = p.transpose(-1, -2) @ do16
    dp = do16 @ vv.transpose(-1, -2)
    delta = (do16 * o).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    ds = torch.nan_to_num(ds, nan=0.0)
    dq16 = (ds @ kk) * f["scale"]
    dk16 = (ds.transpose(-1, -2) @ q16.double()) * f["scale"]

    def reduce_kv(g):
        return g if Hkv == Hq else g.view(B, Hkv, Hq // Hkv, *g.shape[2:]).sum(2)

    two = lambda ex: torch.ldexp(torch.ones(()), ex.double())[..., None, None]
    # |dS| with the magnitudes its rounding errors scale with: P times (|dP| + sum_d |dO16| |O|), plus the
    # absolute error of fp16 rounding near zero: P and dS below fp16's smallest subnormal (2^-24) round to
    # zero in an fp16 pipeline (this build's and the reference's alike), an absolute 2^-25 per element,
    # which the sub_* terms carry in units of 2^-24 (keys / queries that are all but never attended)
    dsa = p * (dp.abs() + (do16.abs() * o.abs()).sum(-1, keepdim=True))
    dsa_sub = dp.abs() + (do16.abs() * o.abs()).sum(-1, keepdim=True) + 1.0
    dq = bf16_rn(dq16 * two(a - G))
    dk = bf16_rn(reduce_kv(dk16) * two(-a - G))
    dv = bf16_rn(reduce_kv(dv16) * two(-ev - G))
    return {"dq": dq, "dk": dk, "dv": dv, "G": G, "a": a, "ev": ev, "out": f["out"], "lse": f["lse"],
            "do16": do16, "delta": delta, "dq16": dq16, "dk16": reduce_kv(dk16), "dv16": reduce_kv(dv16),
            "abs_dq": (dsa @ kk.abs()) * f["scale"] * two(a - G),
            "abs_dk": reduce_kv(dsa.transpose(-1, -2) @ q16.double().abs()) * f["scale"] * two(-a - G),
            "abs_dv": reduce_kv(p.transpose(-1, -2) @ do16.abs()) * two(-ev - G),
            "sub_dq": (dsa_sub @ kk.abs()) * f["scale"] * two(a - G),
            "sub_dk": reduce_kv(dsa_sub.transpose(-1, -2) @ q16.double().abs()) * f["scale"] * two(-a - G),
            "sub_dv": reduce_kv(torch.ones_like(p).transpose(-1, -2) @ do16.abs()) * two(-ev - G)}


# ----------------------------------------------------------------------------- GEMMs

def linear_fused(x, w16, ws, bias=None, target_exp=15, l1=False):
    """Fused inference linear, tbf16/csrc/gemm_sm75.cu:257-284 (kernel :78-226), fp64 accumulation.
    x bf16 (M, K); w16 fp16 (N, K); ws fp32 (N,); bias bf16 (N,) or None -> (y bf16 (M, N), s_inv)."""
    x, w16, ws = _cpu(x), _cpu(w16).contiguous(), _cpu(ws).float().contiguous()
    assert x.dtype == torch.bfloat16 and x.stride(1) == 1 and w16.dtype == torch.float16
    M, K = x.shape
    N = w16.shape[0]
    b = None if bias is None else _cpu(bias).contiguous()
    y = torch.empty((M, N), dtype=torch.bfloat16)
    s_inv = torch.empty(M, dtype=torch.float32)
    lib().orc_linear_fused(_p(x), M, K, x.stride(0), _p(w16), N, K, _p(ws), _p(b), target_exp, int(l1), _p(y), N,
                           _p(s_inv))
    return y, s_inv


# ----------------------------------------------------------------------------- producer fusion
# No reference kernel exists for these (the reference runs the model's torch activation / norm and then
# its row pass, tbf16/ops.py:74-89 and tbf16/csrc/gemm_sm75.cu:27-47); restated here as the bf16 model
# arithmetic followed by the fused rule's row scale and fp16 rounding.

def glu_rows(gate, up, act="silu", target_exp=15):
    """h = bf16(bf16(act(g)) * u) in fp32 (act: silu g / (1 + exp(-g)), or the tanh-approximated GELU),
    then row_scale_fused(h) and h16 = fp16(h / s_inv). Returns (h16, s_inv, h)."""
    g, u = _cpu(gate).float(), _cpu(up).float()
    if act == "silu":
        a = g / (1.0 + torch.exp(-g))
    else:
        a = 0.5 * g * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (g + 0.044715 * g * g * g)))
    h = bf16_rn(bf16_rn(a).float() * u)
    s_inv = row_scale_fused(h, target_exp)
    return f16_rn(h.float() / s_inv[:, None]), s_inv, h


def rmsnorm_rows(x, weight, eps=1e-6, offset=1.0, style="gemma", target_exp=15):
    """r = bf16((x * rsqrt(mean x^2 + eps)) * (w + offset)) ("gemma") or bf16(w * bf16(x * rsqrt(...)))
    ("llama"), fp32 arithmetic, then row_scale_fused(r) and r16 = fp16(r / s_inv). Returns (r16, s_inv, r)."""
    xf, w = _cpu(x).float(), _cpu(weight).float()
    rs = torch.rsqrt((xf * xf).mean(-1, keepdim=True) + eps)
    if style == "gemma":
        r = bf16_rn((xf * rs) * (w + offset))
    else:
        r = bf16_rn(w * bf16_rn(xf * rs).float())
    s_inv = row_scale_fused(r, target_exp)
    return f16_rn(r.float() / s_inv[:, None]), s_inv, r


def add_rmsnorm_rows(x, residual, weight, post_weight=None, eps=1e-6, offset=1.0, style="gemma", target_exp=15):
    """s = bf16(residual + (rmsnorm_rows(x, post_weight)'s bf16 rows if post_weight is given else x)) -- a
    model's bf16 residual add -- then rmsnorm_rows(s, weight). Returns (s, r16, s_inv)."""
    a = _cpu(x)
    if post_weight is not None:
        a = rmsnorm_rows(a, post_weight, eps, offset, style, target_exp)[2]
    s_ = bf16_rn(_cpu(residual).float() + a.float())
    r16, s_inv, _ = rmsnorm_rows(s_, weight, eps, offset, style, target_exp)
    return s_, r16, s_inv


def rope(y, cos, sin):
    """Rotate-half rotary embedding on bf16 tensors, a model's three roundings:
    bf16(bf16(y cos) + bf16(rot(y) sin)), rot(y) = (-y[..., D/2:], y[..., :D/2]); y (..., S, H, D) with
    cos / sin (S, D) broadcast over the heads."""
    y = _cpu(y).float()
    D = y.shape[-1]
    rot = torch.cat([-y[..., D // 2:], y[..., :D // 2]], -1)
    c, s_ = _cpu(cos).float()[:, None, :], _cpu(sin).float()[:, None, :]
    return bf16_rn(bf16_rn(y * c).float() + bf16_rn(rot * s_).float())


def glu_bwd(dh, gate, up, act="silu"):
    """Gradients of h = bf16(act(g)) * u as torch's autograd takes them on bf16 tensors, fp32 arithmetic:
    a = bf16(act(g)), du = bf16(dh a), da = bf16(dh u), dg = bf16(da act'(g)) (silu: s (1 + g (1 - s)),
    s = 1 / (1 + e^-g); tanh-GELU: 0.5 (1 + t) + 0.5 g (1 - t^2) sqrt(2/pi) (1 + 3 0.044715 g^2)).
    Returns (dg, du)."""
    d, g, u = _cpu(dh).float(), _cpu(gate).float(), _cpu(up).float()
    if act == "silu":
        sg = 1.0 / (1.0 + torch.exp(-g))
        a = g / (1.0 + torch.exp(-g))
        dact = sg * (1.0 + g * (1.0 - sg))
    else:
        kb = math.sqrt(2.0 / math.pi)
        t = torch.tanh(kb * (g + 0.044715 * g * g * g))
        a = 0.5 * g * (1.0 + t)
        dact = 0.5 * (1.0 + t) + 0.5 * g * (1.0 - t * t) * kb * (1.0 + 3.0 * 0.044715 * g * g)
    du = bf16_rn(d * bf16_rn(a).float())
    da = bf16_rn(d * u)
    return bf16_rn(da.float() * dact), du


# ----------------------------------------------------------------------------- scaled convolutions

def conv_sample_exp(x: torch.Tensor, target_exp: int) -> torch.Tensor:
    """Per-sample exponent of tbf16/conv.py:47-48 (_pow2_exponent(amax) - t, a zero sample as max 1)."""
    x = _cpu(x).float()
    amax = x.abs().reshape(x.shape[0], -1).amax(1)
    return torch.frexp(torch.where(amax > 0, amax, torch.ones_like(amax)))[1].int() - target_exp


def conv_scaled(x, w16, ws, bias, stride, padding, dilation, groups, target_exp):
    """tbf16/conv.py:34-60 restated with fp64 accumulation: x16 = fp16(x * 2^-e[b]) (exact power-of-two
    scale, C rounding), the convolution of x16 with w16 in fp64, y = bf16((acc * 2^e[b]) * ws[o] + bias[o]).
    Zero padding. Returns (y bf16, acc fp64 of |x16| * |w16| times the scales, for the tolerance)."""
    x, w16 = _cpu(x), _cpu(w16)
    nd = x.dim() - 2
    conv = {1: torch.nn.functional.conv1d, 2: torch.nn.functional.conv2d, 3: torch.nn.functional.conv3d}[nd]
    e = conv_sample_exp(x, target_exp).double()
    bshape = (-1,) + (1,) * (nd + 1)
    x16 = f16_rn((x.double() * torch.exp2(-e).view(bshape)).float())
    acc = conv(x16.double(), w16.double(), None, stride, padding, dilation, groups)
    absacc = conv(x16.double().abs(), w16.double().abs(), None, stride, padding, dilation, groups)
    oshape = (1, -1) + (1,) * nd
    sc = torch.exp2(e).view(bshape) * _cpu(ws).double().view(oshape)
    y = acc * sc
    if bias is not None:
        y = y + _cpu(bias).double().view(oshape)
    return bf16_rn(y), absacc * sc.abs()


def gemm_f16(a16, a_mn, b16, b_mn, M, N, K, sa, sb=None, bias=None):
    """y = bf16((sum_k A[m,k] B[n,k]) * sa[m] * sb[n] + bias[n]) with fp64 accumulation: the
    contraction of ops.py:167-178 (linear_q) and autograd.py:114-120 (_scaled_mm) without the fp16
    rounding of the product. A is a16 (M, K) (a_mn=0) or a16 (K, M) (a_mn=1); B likewise."""
    a16, b16 = _cpu(a16).contiguous(), _cpu(b16).contiguous()
    sa = _cpu(sa).float().contiguous()
    sb = None if sb is None else _cpu(sb).float().contiguous()
    b = None if bias is None else _cpu(bias).contiguous()
    y = torch.empty((M, N), dtype=torch.bfloat16)
    lib().orc_gemm_f16(_p(a16), int(a_mn), a16.stride(0), _p(b16), int(b_mn), b16.stride(0), M, N, K, _p(sa),
                       _p(sb), _p(b), _p(y), N)
    return y


def bf16_trunc(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by truncation. Triton's CPU interpreter (TRITON_INTERPRET=1) casts this way where
    a GPU rounds to nearest; only the golden-vector pins use it."""
    a = _cpu(x).float().contiguous()
    return (a.view(torch.int32) & ~0xFFFF).view(torch.float32).bfloat16()


def linear_small_m_ref(x, w16, ws, bias=None, rounding="rn"):
    """The reference's default inference path for 2 <= M < 256 (tbf16/ops.py:163-164,167-178 with
    small_kernels.cu:35-103): L1 rows at t=15, fp16 GEMM output (rounded to fp16 from an fp64
    accumulation here), then bf16((c16 * sa) * sb + bias). Used only to pin the oracle against
    the reference's own CPU/Triton run (rounding="trunc" reproduces the interpreter's cast)."""
    x16, sx = quantize_rows(x, 15, l1=True)
    acc = x16.double() @ _cpu(w16).double().t()
    c16 = f16_rn(acc.float()).float()
    v = (c16 * sx[:, None]) * _cpu(ws).float()[None, :]
    if bias is not None:
        v = v + _cpu(bias).float()[None, :]
    return bf16_trunc(v) if rounding == "trunc" else bf16_rn(v)


def gemv_ref(x, w16, ws, bias=None):
    """The reference's single-row linear (tbf16/csrc/small_kernels.cu:107-132): fp32 products of bf16 x and
    fp16 w summed, times ws, plus bias, rounded to bf16 once. Summed in fp64 here; the kernel's fp32 sum
    order differs, so results agree to a bf16 ulp (plus fp32 rounding under cancellation)."""
    v = _cpu(x).double() @ _cpu(w16).double().t() * _cpu(ws).double()[None, :]
    if bias is not None:
        v = v + _cpu(bias).double()[None, :]
    return bf16_rn(v.float())


def linear_train(x, w, bias, dy, rows=None, dw_rows=None):
    """tbf16/autograd.py:58-90 (ScaledLinearFn) with this build's GEMM semantics (fp32/fp64
    accumulation, one bf16 rounding). Exponent conventions kept from the reference:
      forward: x rows max t=_target_exp(K) (ops.py:133-137), w rows t=_target_exp(K) (ops.py:140-142)
      dX:      dy rows L1 t=15 (autograd.py:79), w columns t=_target_exp(N) (autograd.py:80)
      dW:      dy columns t=min(0, 15 - ceil(log2 M)) with row_mul = sx (autograd.py:85-87)
      db:      fp32 column sum of dy (autograd.py:88-89), here summed in fp64.
    x (M, K), w (N, K), bias (N,) or None, dy (M, N), all bf16.

    rows / dw_rows (optional index tensors): the scales are always computed from the full operands,
    but y and dx are returned only for rows `rows` of M and dw only for rows `dw_rows` of N, so that
    full-size layers can be checked on a sample of their outputs."""
    x2, w, dy2 = _cpu(x).reshape(-1, x.shape[-1]).contiguous(), _cpu(w).contiguous(), _cpu(dy).reshape(-1, w.shape[0]).contiguous()
    M, K = x2.shape
    N = w.shape[0]
    rows = torch.arange(M) if rows is None else _cpu(rows).long()
    dw_rows = torch.arange(N) if dw_rows is None else _cpu(dw_rows).long()
    t = target_exp(K)
    x16, sx = quantize_rows(x2, t)
    w16, sw = quantize_rows(w, t)
    y = gemm_f16(x16[rows], 0, w16, 0, len(rows), N, K, sx[rows], sw, bias)
    dy16, sdy = quantize_rows(dy2, 15, l1=True)
    w16c, swc = quantize_cols(w, target_exp(N))
    dx = gemm_f16(dy16[rows], 0, w16c, 1, len(rows), K, N, sdy[rows], swc)
    t2 = min(0, 15 - math.ceil(math.log2(max(M, 1))))
    dy16c, sdyc = quantize_cols(dy2, t2, row_mul=sx)
    dw = gemm_f16(dy16c[:, dw_rows], 1, x16, 1, len(dw_rows), K, M, sdyc[dw_rows], None)
    db = None if bias is None else bf16_rn(dy2.double().sum(0))
    return {"y": y, "dx": dx, "dw": dw, "db": db, "x16": x16, "sx": sx, "w16": w16, "sw": sw, "dy16": dy16,
            "sdy": sdy, "w16c": w16c, "swc": swc, "dy16c": dy16c, "sdyc": sdyc, "rows": rows, "dw_rows": dw_rows}


def rel_err(y, ref):
    y, ref = _cpu(y).double(), _cpu(ref).double()
    return ((y - ref).norm() / ref.norm()).item()


def bf16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 numbers at |v| (fp64 tensor): 2^(floor(log2|v|) - 7), min normal spacing below."""
    a = _cpu(v).double().abs().clamp_min(2.0 ** -126)
    return torch.ldexp(torch.ones_like(a), (torch.floor(torch.log2(a)) - 7).to(torch.int32))


def to_u16(t: torch.Tensor) -> np.ndarray:
    return _cpu(t).contiguous().view(torch.int16).numpy().view(np.uint16)


if os.environ.get("TBF16_ORACLE_BUILD_ON_IMPORT"):
    lib()


# ----------------------------------------------------------------------------- attention dropout mask

def _fmix32(x: np.ndarray) -> np.ndarray:
    """murmur3's 32-bit finaliser on uint32 arrays (wrapping arithmetic)."""
    x = x.astype(np.uint32)
    x ^= x >> np.uint32(16)
    x = (x * np.uint32(0x85EBCA6B)).astype(np.uint32)
    x ^= x >> np.uint32(13)
    x = (x * np.uint32(0xC2B2AE35)).astype(np.uint32)
    x ^= x >> np.uint32(16)
    return x


def dropout_params(p: float):
    """(threshold, 1 / keep probability): a key is kept when its 16 hash bits are >= round(p * 65536)."""
    thr = int(round(p * 65536.0))
    return thr, 65536.0 / (65536 - thr)


def dropout_keep(seed: int, BH: int, Sq: int, Sk: int, p: float) -> torch.Tensor:
    """bool (BH, Sq, Sk) keep mask of this build's attention dropout (no counterpart in the reference,
    whose dropout is torch's Philox stream): row key = fmix32((fmix32(bh ^ seed_lo) + i * 0x9e3779b9) ^
    seed_hi), pair bits = fmix32(row key ^ (j / 2) * 0x7feb352d), key j takes the low (even j) or high (odd j)
    16 bits, kept when >= round(p * 65536). Restated here so the GPU's mask can be checked bit for bit."""
    with np.errstate(over="ignore"):
        thr, _ = dropout_params(p)
        s_lo, s_hi = np.uint32(seed & 0xFFFFFFFF), np.uint32((seed >> 32) & 0xFFFFFFFF)
        bh = np.arange(BH, dtype=np.uint32)[:, None]
        i = np.arange(Sq, dtype=np.uint32)[None, :]
        rk = _fmix32(((_fmix32(bh ^ s_lo) + (i * np.uint32(0x9E3779B9)).astype(np.uint32)).astype(np.uint32)) ^ s_hi)
        j = np.arange(Sk, dtype=np.uint32)
        jp = ((j >> np.uint32(1)) * np.uint32(0x7FEB352D)).astype(np.uint32)
        bits = _fmix32(rk[:, :, None] ^ jp[None, None, :])
        half = np.where((j & 1) == 1, bits >> np.uint32(16), bits & np.uint32(0xFFFF))
        return torch.from_numpy(half >= thr)
