"""bf16 matmuls on fp16 tensor cores with exact power-of-two scaling, on B200 (sm_100a).

Same public surface as the reference's tbf16/ops.py (quantize_rows, prepare_weight, scaled_linear,
linear_q, small_m_linear, quantize_rows_shared, _target_exp), plus linear_host for activations that
live in pinned host memory and the producer-fused glu_rows / rmsnorm_rows / add_rmsnorm_rows
(glu_linear, rmsnorm_linear), which compute a linear's row scales in the kernel that produces its input,
rmsnorm (with an optional residual add), rmsnorm_rope (QK-norm + rotary embedding in one pass) and
glu_bwd (the gated activation's backward for training). The work runs in libtbf16_sm100.so: a
row-amax -> exponent pass (which
also writes the fp16 copy of x for large N) and a warp-specialised TMA + tcgen05 GEMM that
accumulates in fp32 in TMEM and writes bf16 straight from the accumulator. Up to 4 rows take a
weight-streaming kernel instead (the reference's single-row GEMV, extended), up to 256 rows a split-K
variant of the GEMM that keeps the whole GPU streaming the weight. The reference's Triton
kernels and its cuBLAS small-M branch are gone, and there is no CPU fallback.
"""
import math
import os
import weakref

import torch

from ._ext import available, call, ptr, require_cuda, stream_ptr

# Kept for callers that set them (reference tbf16/ops.py:19-23); this build has one path for every M.
_USE_CUDA = os.environ.get("TBF16_BACKEND", "cuda") == "cuda"
_GEMM = os.environ.get("TBF16_GEMM", "")
FUSED_MIN_M = 1
# Row scaling of the fused GEMM: row max -> [2^14, 2^15) (reference tbf16/ops.py:24-26).
_FUSED_SCALE = (15, False)
# Rows scaled by their L1 norm for the training dX GEMM (reference tbf16/ops.py:129-130).
L1_TARGET = 15
SMALL_M = 2
GEMV_ROWS = 4  # rows taken by the weight-streaming kernel (it accepts up to TBF16_GEMV_MAX_ROWS = 8;
               # from 5 rows on the skinny GEMM streams the weight faster)
SKINNY_ROWS = 256  # rows handled by the split-K skinny GEMM (kSkinnyMaxRows in the library)


def _target_exp(K: int) -> int:
    """Rows are scaled to amax in [2^(t-1), 2^t) so that an fp16 product of K terms stays below
    K * 4^t <= 65504; t = 0 covers K <= 32768 (reference tbf16/ops.py:29-32)."""
    return min(0, (15 - math.ceil(math.log2(max(K, 1)))) // 2)


def _check_bf16_2d(x, name):
    require_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise RuntimeError(f"tbf16: {name} must be a 2-D bf16 CUDA tensor, got {x.dtype} {tuple(x.shape)}")


def _rows_ok(t):
    return t.stride(-1) == 1 and t.shape[-1] % 8 == 0 and t.stride(0) % 8 == 0 and t.data_ptr() % 16 == 0


def quantize_rows(x: torch.Tensor, target_exp: int = 0, l1: bool = False):
    """bf16 (R, K) -> (fp16 (R, K), fp32 (R,) inverse scales). Lossless for normal bf16 values inside
    fp16's range after scaling. Each row's max (or with l1=True its L1 norm) goes to [2^(t-1), 2^t)."""
    _check_bf16_2d(x, "x")
    if not _rows_ok(x):
        x = _pad_cols(x)
    R, Kp = x.shape
    y = torch.empty((R, Kp), device=x.device, dtype=torch.float16)
    s_inv = torch.empty((R,), device=x.device, dtype=torch.float32)
    call("tbf16_quantize_rows", ptr(x), R, Kp, x.stride(0), int(target_exp), int(bool(l1)), ptr(y), Kp, ptr(s_inv),
         stream_ptr(x.device))
    return y, s_inv


def _pad_cols(x: torch.Tensor, mult: int = 8) -> torch.Tensor:
    """Contiguous copy with the last dimension zero-padded to a multiple of `mult` (16-byte rows)."""
    K = x.shape[-1]
    Kp = (K + mult - 1) // mult * mult
    out = torch.zeros((*x.shape[:-1], Kp), device=x.device, dtype=x.dtype)
    out[..., :K] = x
    return out


class _RowCache:
    """Reuses quantize_rows results when the same activation feeds several linear layers
    (Q/K/V, gate/up). Keyed by tensor identity through a weakref plus the version counter, so
    freed or modified tensors never hit (reference tbf16/ops.py:107-123)."""

    def __init__(self, size=8):
        self.size, self.entries = size, []

    def get(self, x, t, make):
        for ref, ver, tt, val in self.entries:
            if ref() is x and ver == x._version and tt == t:
                return val
        val = make()
        self.entries.append((weakref.ref(x), x._version, t, val))
        if len(self.entries) > self.size:
            self.entries.pop(0)
        return val


_row_cache = _RowCache()


def quantize_rows_shared(x: torch.Tensor, l1: bool = False):
    """quantize_rows of x viewed as (-1, K), shared across calls on the same tensor."""
    K = x.shape[-1]
    t = L1_TARGET if l1 else _target_exp(K)
    return _row_cache.get(x, (t, l1), lambda: quantize_rows(x.reshape(-1, K).contiguous(), t, l1))


def prepare_weight(w: torch.Tensor):
    """nn.Linear weight (N, K) bf16 -> (fp16 (N, K), fp32 (N,) inverse scales). Do this once."""
    return quantize_rows(w.contiguous(), _target_exp(w.shape[1]))


def _bias_ok(bias, N, device):
    if bias is None:
        return None
    require_cuda(bias)
    if bias.dtype != torch.bfloat16:
        bias = bias.to(torch.bfloat16)
    bias = bias.contiguous()
    if bias.numel() != N:
        raise RuntimeError(f"tbf16: bias has {bias.numel()} elements, expected {N}")
    return bias


def _materialise(M, N, K) -> bool:
    """Whether the linear should write an fp16 copy of x in its row pass (TBF16_LINEAR=fused forces
    the in-GEMM conversion, =materialise the copy). The in-GEMM conversion is redone once per 256-wide
    N tile, so it only pays when N fits in one or two tiles; up to 256 rows the copy is small and the
    split-K skinny GEMM (fp16 operands only) takes the product."""
    mode = os.environ.get("TBF16_LINEAR", "")
    if mode == "fused":
        return False
    if mode == "materialise":
        return True
    return N > 512 or M <= SKINNY_ROWS


@torch.autocast("cuda", enabled=False)
def scaled_linear(x: torch.Tensor, w16: torch.Tensor, w_sinv: torch.Tensor, bias=None):
    """y = x @ W^T + b for bf16 x, with W given by prepare_weight. Returns bf16.

    Routed by the number of rows M (reference fused path, gemm_sm75.cu:257-284, for every M): up to
    GEMV_ROWS rows, one weight-streaming pass (tbf16_gemv); otherwise tbf16_linear: the row pass
    computes each row's power-of-two scale and, when _materialise says so (N above 512 or at most
    SKINNY_ROWS rows), also writes fp16(x * 2^s) in the same read of x, and the tcgen05 GEMM then
    runs on fp16 operands (split-K skinny GEMM up to SKINNY_ROWS rows, CTA-pair or single-CTA GEMM
    above); for narrow N the GEMM's converter warps build the fp16 tile from bf16 x in shared memory
    instead. The product leaves the fp32 accumulator as bf16 once."""
    require_cuda(x, w16, w_sinv)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"tbf16.scaled_linear: x must be bf16, got {x.dtype}")
    if w16.dtype != torch.float16 or w16.dim() != 2:
        raise RuntimeError("tbf16.scaled_linear: w16 must be fp16 (N, K) from prepare_weight")
    shape = x.shape
    K = shape[-1]
    N = w16.shape[0]
    if w16.shape[1] < K or w_sinv.numel() != N:
        raise RuntimeError(f"tbf16.scaled_linear: weight {tuple(w16.shape)} does not match K={K}")
    x2 = x.reshape(-1, K)
    if not _rows_ok(x2):
        x2 = _pad_cols(x2) if K % 8 else x2.contiguous()
    if not _rows_ok(w16) or w16.shape[1] != x2.shape[1]:
        w16 = _pad_cols(w16[:, :K]) if K % 8 else w16.contiguous()
    M, Kp = x2.shape
    if M <= GEMV_ROWS:  # decode: one pass over the weight for all rows
        return _gemv(x2, w16, w_sinv, _bias_ok(bias, N, x.device), N).reshape(*shape[:-1], N)
    Np = (N + 7) // 8 * 8
    b = _bias_ok(bias, N, x.device)
    ws = w_sinv.contiguous().float()
    if Np != N:  # the GEMM writes 16-byte rows: pad the output columns and slice them off
        w16 = torch.cat([w16, w16.new_zeros(Np - N, w16.shape[1])])
        ws = torch.cat([ws, ws.new_ones(Np - N)])
        b = None if b is None else torch.cat([b, b.new_zeros(Np - N)])
    y = torch.empty((M, Np), device=x.device, dtype=torch.bfloat16)
    s_inv = torch.empty((M,), device=x.device, dtype=torch.float32)
    # fp16 copy of x written by the row pass (one read of x); the GEMM then runs on fp16 operands
    x16 = torch.empty((M, Kp), device=x.device, dtype=torch.float16) if _materialise(M, Np, Kp) else None
    t, l1 = _FUSED_SCALE
    call("tbf16_linear", ptr(x2), M, Kp, x2.stride(0), ptr(w16), Np, w16.stride(0), ptr(ws), ptr(b), ptr(y), Np,
         ptr(s_inv), ptr(x16), t, int(l1), stream_ptr(x.device))
    if Np != N:
        y = y[:, :N]
    return y.reshape(*shape[:-1], N)


def linear_host(x_host: torch.Tensor, w16: torch.Tensor, w_sinv: torch.Tensor, bias=None, out=None,
                chunk_rows: int = 1024) -> torch.Tensor:
    """scaled_linear for activations in pinned host memory: y_host (M, N) bf16 = x_host @ W^T + b.

    Rows go through in chunks on three streams, so the upload of chunk c+1, the linear of chunk c and
    the download of chunk c-1 overlap (PCIe copies in both directions run on separate copy engines);
    two device buffers per direction. Returns `out` (pinned, allocated if None) once the last chunk's
    download is enqueued: it is complete when the current stream reaches this point (synchronise
    before reading it on the host). Same arithmetic as scaled_linear on each row."""
    if x_host.is_cuda or x_host.dtype != torch.bfloat16 or x_host.dim() != 2:
        raise RuntimeError("tbf16.linear_host: x_host must be a 2-D bf16 tensor in host memory")
    require_cuda(w16, w_sinv)
    M, K = x_host.shape
    N = w16.shape[0]
    dev = w16.device
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, pin_memory=True)
    if M == 0:
        return out
    if K % 8 or N % 8 or w16.shape[1] != K or w16.stride(0) != K:
        raise RuntimeError("tbf16.linear_host: K and N must be multiples of 8 (use scaled_linear)")
    cur = torch.cuda.current_stream(dev)
    rows = max(1, min(chunk_rows, M))
    up, down, xb, yb, s_inv, x16 = _host_pipeline(dev, cur, rows, K, N)
    ws = w_sinv.contiguous().float()
    bb = _bias_ok(bias, N, dev)
    t, l1 = _FUSED_SCALE
    sp = stream_ptr(dev)
    uploaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    downloaded = [torch.cuda.Event() for _ in range(2)]
    start = torch.cuda.Event()
    start.record(cur)
    up.wait_event(start)
    down.wait_event(start)
    for c, (r0, n) in enumerate(_host_chunks(M, rows)):
        b = c & 1
        with torch.cuda.stream(up):
            if c >= 2:
                up.wait_event(computed[b])  # the linear of chunk c-2 has read this x buffer
            xb[b][:n].copy_(x_host[r0:r0 + n], non_blocking=True)
            uploaded[b].record(up)
        cur.wait_event(uploaded[b])
        if c >= 2:
            cur.wait_event(downloaded[b])  # chunk c-2's result has left this y buffer
        if n <= GEMV_ROWS:
            yb[b][:n] = _gemv(xb[b][:n], w16, w_sinv, bb, N)
        else:
            call("tbf16_linear", ptr(xb[b]), n, K, K, ptr(w16), N, K, ptr(ws), ptr(bb), ptr(yb[b]), N, ptr(s_inv),
                 ptr(x16), t, int(l1), sp)
        computed[b].record(cur)
        with torch.cuda.stream(down):
            down.wait_event(computed[b])
            out[r0:r0 + n].copy_(yb[b][:n], non_blocking=True)
            downloaded[b].record(down)
    cur.wait_stream(down)
    return out


def _host_chunks(M, rows):
    """(first row, rows) of linear_host's chunks: full `rows` chunks, except that the first and the last
    are split into a quarter and three quarters, so that the first upload and the last download, which
    nothing overlaps, are short."""
    if M <= rows:
        return [(0, M)]
    q = max(8, rows // 4)
    sizes = [q, rows - q]
    left = M - rows
    while left > rows + q:
        sizes.append(rows)
        left -= rows
    sizes += [left - q, q] if left > q else [left]
    out, r0 = [], 0
    for n in sizes:
        out.append((r0, n))
        r0 += n
    return out


# Copy streams and chunk buffers of linear_host, kept per (device, calling stream, shape): calls on one
# stream are ordered (each waits for the previous call's downloads), so they can share the buffers,
# and nothing is freed while the copy streams may still use it.
_HOST_PIPES = {}


def _host_pipeline(dev, cur, rows, K, N):
    key = (dev.index, cur.cuda_stream, rows, K, N)
    pipe = _HOST_PIPES.get(key)
    if pipe is None:
        if len(_HOST_PIPES) >= 8:  # drop the cache, once its copy streams are idle
            for old in _HOST_PIPES.values():
                old[0].synchronize()
                old[1].synchronize()
            _HOST_PIPES.clear()
        pipe = (torch.cuda.Stream(dev), torch.cuda.Stream(dev),
                [torch.empty((rows, K), device=dev, dtype=torch.bfloat16) for _ in range(2)],
                [torch.empty((rows, N), device=dev, dtype=torch.bfloat16) for _ in range(2)],
                torch.empty((rows,), device=dev, dtype=torch.float32),
                torch.empty((rows, K), device=dev, dtype=torch.float16) if _materialise(rows, N, K) else None)
        _HOST_PIPES[key] = pipe
    return pipe


def _gemm_f16(a16, a_mn, b16, b_mn, M, N, K, sa, sb=None, bias=None):
    """y (M, N) bf16 = (A @ B^T) * sa[:, None] * sb[None, :] + bias on the tcgen05 GEMM.
    A = a16 (M, K) or, with a_mn, a16 (K, M); B = b16 (N, K) or, with b_mn, b16 (K, N)."""
    require_cuda(a16, b16, sa)
    dev = a16.device
    y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
    sa = sa.contiguous().float()
    sb = None if sb is None else sb.contiguous().float()
    call("tbf16_gemm_f16", ptr(a16), int(a_mn), a16.stride(0), ptr(b16), int(b_mn), b16.stride(0), M, N, K, ptr(sa),
         ptr(sb), ptr(bias), ptr(y), N, stream_ptr(dev))
    return y


@torch.autocast("cuda", enabled=False)
def linear_q(x16, x_sinv, w16, w_sinv, bias=None):
    """GEMM + epilogue on already-quantized rows: (x16 * x_sinv) @ (w16 * w_sinv)^T + bias, bf16 (M, N).
    The product goes from the fp32 accumulator to bf16 once (the reference rounds it to fp16 first,
    reference tbf16/ops.py:167-178)."""
    require_cuda(x16, w16)
    M, K = x16.shape
    N = w16.shape[0]
    b = _bias_ok(bias, N, x16.device)
    if K % 8 or N % 8 or not _rows_ok(x16) or not _rows_ok(w16):
        return (_gemm_padded(x16, x_sinv, w16, w_sinv, b))
    return _gemm_f16(x16, 0, w16, 0, M, N, K, x_sinv, w_sinv, b)


def _gemm_padded(x16, x_sinv, w16, w_sinv, b):
    M, K = x16.shape
    N = w16.shape[0]
    Np = (N + 7) // 8 * 8
    xp, wp = _pad_cols(x16), _pad_cols(w16)
    ws = w_sinv.contiguous().float()
    if Np != N:
        wp = torch.cat([wp, wp.new_zeros(Np - N, wp.shape[1])])
        ws = torch.cat([ws, ws.new_ones(Np - N)])
        b = None if b is None else torch.cat([b, b.new_zeros(Np - N)])
    return _gemm_f16(xp, 0, wp, 0, M, Np, xp.shape[1], x_sinv, ws, b)[:, :N]


def _gemv(x2, w16, w_sinv, b, N):
    """y (M, N) bf16 for M <= GEMV_ROWS rows: fp32 products of bf16 x and fp16 w, times w_sinv, plus bias
    (the reference's single-row kernel, small_kernels.cu:107-132), one pass over the weight."""
    M, K = x2.shape
    y = torch.empty((M, N), device=x2.device, dtype=torch.bfloat16)
    ws = w_sinv.contiguous().float()
    call("tbf16_gemv", ptr(x2), M, K, x2.stride(0), ptr(w16), N, w16.stride(0), ptr(ws), ptr(b), ptr(y), N,
         stream_ptr(x2.device))
    return y


_ACTS = {"silu": 0, "gelu_tanh": 1}
_NORM_STYLES = {"gemma": 0, "llama": 1}


def _rows2d(t, name):
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"tbf16.{name}: expected bf16, got {t.dtype}")
    t2 = t.reshape(-1, t.shape[-1])
    return t2 if _rows_ok(t2) else t2.contiguous()


@torch.autocast("cuda", enabled=False)
def glu_rows(gate: torch.Tensor, up: torch.Tensor, act: str = "silu", target_exp: int = 15, want_h: bool = False):
    """Producer-fused gated activation: h = bf16(bf16(act(gate)) * up) (torch's act(g) * u on bf16 tensors,
    to within one bf16 ulp)
    with the row scales of the fused linear computed in the same pass. Returns (h16, s_inv[, h]): the fp16
    operand fp16(h / s_inv) and the fp32 power-of-two inverse row scales, as quantize_rows / row_scale
    give for h. act: "silu" or "gelu_tanh"."""
    require_cuda(gate, up)
    if act not in _ACTS:
        raise RuntimeError(f"tbf16.glu_rows: act must be one of {sorted(_ACTS)}")
    if gate.shape != up.shape:
        raise RuntimeError("tbf16.glu_rows: gate and up shapes differ")
    g2, u2 = _rows2d(gate, "glu_rows"), _rows2d(up, "glu_rows")
    M, I = g2.shape
    if I % 8:
        raise RuntimeError("tbf16.glu_rows: the row length must be a multiple of 8")
    h16 = torch.empty((M, I), device=gate.device, dtype=torch.float16)
    s_inv = torch.empty((M,), device=gate.device, dtype=torch.float32)
    h = torch.empty((M, I), device=gate.device, dtype=torch.bfloat16) if want_h else None
    call("tbf16_glu_rows", ptr(g2), g2.stride(0), ptr(u2), u2.stride(0), M, I, _ACTS[act], int(target_exp), ptr(h16), I,
         ptr(s_inv), ptr(h), I, stream_ptr(gate.device))
    shape = gate.shape
    out = (h16.reshape(shape), s_inv.reshape(shape[:-1]))
    return out + (h.reshape(shape),) if want_h else out


def glu_bwd(dh: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, act: str = "silu"):
    """Gradients of h = bf16(act(gate)) * up as torch's autograd gives them on bf16 tensors (to within one
    bf16 ulp), in one pass:
    returns (d_gate, d_up), bf16 of gate's shape."""
    require_cuda(dh, gate, up)
    if act not in _ACTS:
        raise RuntimeError(f"tbf16.glu_bwd: act must be one of {sorted(_ACTS)}")
    if not (dh.shape == gate.shape == up.shape):
        raise RuntimeError("tbf16.glu_bwd: dh, gate and up shapes differ")
    h2, g2, u2 = (_rows2d(t, "glu_bwd") for t in (dh, gate, up))
    M, I = g2.shape
    if I % 8:
        raise RuntimeError("tbf16.glu_bwd: the row length must be a multiple of 8")
    dg = torch.empty((M, I), device=gate.device, dtype=torch.bfloat16)
    du = torch.empty((M, I), device=gate.device, dtype=torch.bfloat16)
    call("tbf16_glu_bwd", ptr(h2), h2.stride(0), ptr(g2), g2.stride(0), ptr(u2), u2.stride(0), M, I, _ACTS[act],
         ptr(dg), I, ptr(du), I, stream_ptr(gate.device))
    return dg.reshape(gate.shape), du.reshape(gate.shape)


@torch.autocast("cuda", enabled=False)
def rmsnorm_rows(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, offset: float = 1.0, style: str = "gemma",
                 target_exp: int = 15, want_r: bool = False):
    """Producer-fused RMSNorm with the row scales of the linear that follows. style "gemma":
    r = bf16((x * rsqrt(mean(x^2) + eps)) * (weight + offset)) in fp32; "llama":
    r = bf16(weight * bf16(x * rsqrt(mean(x^2) + eps))). Returns (r16, s_inv[, r]) as glu_rows."""
    require_cuda(x, weight)
    if style not in _NORM_STYLES:
        raise RuntimeError(f"tbf16.rmsnorm_rows: style must be one of {sorted(_NORM_STYLES)}")
    x2 = _rows2d(x, "rmsnorm_rows")
    M, K = x2.shape
    w = weight.to(torch.bfloat16).contiguous()
    if w.numel() != K or K % 8:
        raise RuntimeError("tbf16.rmsnorm_rows: weight must have the row length, a multiple of 8")
    r16 = torch.empty((M, K), device=x.device, dtype=torch.float16)
    s_inv = torch.empty((M,), device=x.device, dtype=torch.float32)
    r = torch.empty((M, K), device=x.device, dtype=torch.bfloat16) if want_r else None
    call("tbf16_rmsnorm_rows", ptr(x2), x2.stride(0), ptr(w), M, K, float(eps), _NORM_STYLES[style], float(offset),
         int(target_exp), ptr(r16), K, ptr(s_inv), ptr(r), K, stream_ptr(x.device))
    out = (r16.reshape(x.shape), s_inv.reshape(x.shape[:-1]))
    return out + (r.reshape(x.shape),) if want_r else out


@torch.autocast("cuda", enabled=False)
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, offset: float = 1.0, style: str = "gemma",
            residual=None):
    """Plain RMSNorm (bf16 in and out) on the rmsnorm_rows kernel, for norms that feed no linear: one read
    of x, one write of the result, the same roundings as rmsnorm_rows. With `residual` (x's shape, bf16):
    residual + rmsnorm(x) in the same pass, as a model adds the two bf16 tensors."""
    require_cuda(x, weight)
    if style not in _NORM_STYLES:
        raise RuntimeError(f"tbf16.rmsnorm: style must be one of {sorted(_NORM_STYLES)}")
    x2 = _rows2d(x, "rmsnorm")
    M, K = x2.shape
    w = weight.to(torch.bfloat16).contiguous()
    if w.numel() != K or K % 8:
        raise RuntimeError("tbf16.rmsnorm: weight must have the row length, a multiple of 8")
    r = torch.empty((M, K), device=x.device, dtype=torch.bfloat16)
    if residual is None:
        call("tbf16_rmsnorm_rows", ptr(x2), x2.stride(0), ptr(w), M, K, float(eps), _NORM_STYLES[style], float(offset),
             15, None, 0, None, ptr(r), K, stream_ptr(x.device))
    else:
        if residual.shape != x.shape:
            raise RuntimeError("tbf16.rmsnorm: residual must have x's shape")
        r2 = _rows2d(residual, "rmsnorm")
        call("tbf16_add_rmsnorm_rows", ptr(x2), x2.stride(0), ptr(r2), r2.stride(0), ptr(w), None, M, K, float(eps),
             _NORM_STYLES[style], float(offset), 15, ptr(r), K, None, 0, None, None, 0, stream_ptr(x.device))
    return r.reshape(x.shape)


@torch.autocast("cuda", enabled=False)
def add_rmsnorm_rows(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, post_weight=None,
                     eps: float = 1e-6, offset: float = 1.0, style: str = "gemma", target_exp: int = 15):
    """A residual block's end and the next block's producer-fused norm in one pass:
    s = residual + (rmsnorm(x, post_weight) if post_weight is given else x)  (bf16, the new residual stream),
    then rmsnorm_rows(s, weight). Returns (s, r16, s_inv) -- s for the next residual add, (r16, s_inv) the
    next linear's fp16 operand and row scales, as rmsnorm_rows."""
    require_cuda(x, residual, weight)
    if style not in _NORM_STYLES:
        raise RuntimeError(f"tbf16.add_rmsnorm_rows: style must be one of {sorted(_NORM_STYLES)}")
    if residual.shape != x.shape:
        raise RuntimeError("tbf16.add_rmsnorm_rows: residual must have x's shape")
    x2, r2 = _rows2d(x, "add_rmsnorm_rows"), _rows2d(residual, "add_rmsnorm_rows")
    M, K = x2.shape
    w = weight.to(torch.bfloat16).contiguous()
    pw = None if post_weight is None else post_weight.to(torch.bfloat16).contiguous()
    if w.numel() != K or K % 8 or (pw is not None and pw.numel() != K):
        raise RuntimeError("tbf16.add_rmsnorm_rows: weights must have the row length, a multiple of 8")
    s = torch.empty((M, K), device=x.device, dtype=torch.bfloat16)
    r16 = torch.empty((M, K), device=x.device, dtype=torch.float16)
    s_inv = torch.empty((M,), device=x.device, dtype=torch.float32)
    call("tbf16_add_rmsnorm_rows", ptr(x2), x2.stride(0), ptr(r2), r2.stride(0), ptr(pw), ptr(w), M, K, float(eps),
         _NORM_STYLES[style], float(offset), int(target_exp), ptr(s), K, ptr(r16), K, ptr(s_inv), None, 0,
         stream_ptr(x.device))
    return s.reshape(x.shape), r16.reshape(x.shape), s_inv.reshape(x.shape[:-1])


@torch.autocast("cuda", enabled=False)
def rmsnorm_rope(x: torch.Tensor, weight, cos: torch.Tensor, sin: torch.Tensor, eps: float = 1e-6, offset: float = 1.0,
                 style: str = "gemma"):
    """Per-head RMSNorm (weight None: none) and rotate-half rotary embedding of x (..., S, H, D) bf16 in one
    pass: rmsnorm(x) * cos + rot(rmsnorm(x)) * sin with torch's bf16 roundings, rot(y) = cat(-y[..., D/2:],
    y[..., :D/2]); cos, sin bf16 holding S x D values (e.g. (S, D) or (1, 1, S, D)). D = 64, 128, 256 or 512.
    Returns a tensor of x's shape (contiguous)."""
    require_cuda(x, cos, sin)
    if x.dtype != torch.bfloat16 or cos.dtype != torch.bfloat16 or sin.dtype != torch.bfloat16 or x.dim() < 3:
        raise RuntimeError("tbf16.rmsnorm_rope: bf16 x (..., S, H, D), cos and sin expected")
    S, H, D = x.shape[-3:]
    if cos.numel() != S * D or sin.numel() != S * D:
        raise RuntimeError("tbf16.rmsnorm_rope: cos / sin must hold S x D values")
    if style not in _NORM_STYLES:
        raise RuntimeError(f"tbf16.rmsnorm_rope: style must be one of {sorted(_NORM_STYLES)}")
    # heads contiguous, tokens a uniform stride apart (e.g. a column slice of a fused QKV output): read in place
    lead = x.shape[:-2]
    tok = x.stride(-3)
    uniform = all(x.stride(i) == tok * math.prod(lead[i + 1:]) for i in range(len(lead)) if lead[i] > 1)
    xc = x if (x.stride(-1) == 1 and x.stride(-2) == D and uniform and tok >= H * D and tok % 8 == 0
               and x.data_ptr() % 16 == 0) else x.contiguous()
    if xc is not x:
        tok = H * D
    c2, s2 = cos.reshape(S, D).contiguous(), sin.reshape(S, D).contiguous()
    w = None if weight is None else weight.to(torch.bfloat16).contiguous()
    out = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
    M = x.numel() // D
    call("tbf16_rmsnorm_rope", ptr(xc), tok, ptr(w), M, D, float(eps), _NORM_STYLES[style], float(offset), ptr(c2),
         ptr(s2), D, S, H, ptr(out), D, stream_ptr(x.device))
    return out


def _linear_from_rows(q16, s_inv, bf16_rows, w16, w_sinv, bias, lead_shape):
    """The down projection of an already row-scaled operand: the same kernels and arithmetic as
    scaled_linear on the bf16 rows (GEMV semantics up to GEMV_ROWS rows, which need the bf16 rows)."""
    K = q16.shape[-1]
    M = q16.numel() // K
    N = w16.shape[0]
    if M <= GEMV_ROWS:
        return scaled_linear(bf16_rows, w16, w_sinv, bias)
    if not _rows_ok(w16) or w16.shape[1] != K or N % 8:
        return scaled_linear(bf16_rows, w16, w_sinv, bias)
    y = _gemm_f16(q16.reshape(M, K), 0, w16, 0, M, N, K, s_inv.reshape(M), w_sinv.contiguous().float(),
                  _bias_ok(bias, N, q16.device))
    return y.reshape(*lead_shape, N)


def glu_linear(gate: torch.Tensor, up: torch.Tensor, w16: torch.Tensor, w_sinv: torch.Tensor, bias=None,
               act: str = "silu"):
    """down(act(gate) * up) for a gated MLP, equal to scaled_linear(act(gate) * up, w16, w_sinv, bias)
    on the bf16 product, without its separate activation and row passes (glu_rows feeds the GEMM)."""
    few = gate.numel() // gate.shape[-1] <= GEMV_ROWS
    res = glu_rows(gate, up, act, want_h=few)
    return _linear_from_rows(res[0], res[1], res[2] if few else None, w16, w_sinv, bias, gate.shape[:-1])


def rmsnorm_linear(x: torch.Tensor, weight: torch.Tensor, w16: torch.Tensor, w_sinv: torch.Tensor, bias=None,
                   eps: float = 1e-6, offset: float = 1.0, style: str = "gemma"):
    """linear(RMSNorm(x)) equal to scaled_linear(rmsnorm(x), ...) on the bf16 normalised rows, with the norm
    and the linear's row pass in one kernel (rmsnorm_rows feeds the GEMM)."""
    few = x.numel() // x.shape[-1] <= GEMV_ROWS
    res = rmsnorm_rows(x, weight, eps, offset, style, want_r=few)
    return _linear_from_rows(res[0], res[1], res[2] if few else None, w16, w_sinv, bias, x.shape[:-1])


def small_m_linear(x2: torch.Tensor, w16: torch.Tensor, w_sinv: torch.Tensor, bias=None):
    """The reference's small-M entry point (reference tbf16/ops.py:207-218): up to GEMV_ROWS rows go
    through the weight-streaming kernel, more through the tcgen05 GEMM (scaled_linear routes the same way)."""
    return scaled_linear(x2, w16, w_sinv, bias)


__all__ = ["quantize_rows", "quantize_rows_shared", "prepare_weight", "scaled_linear", "linear_q", "small_m_linear",
           "linear_host", "glu_rows", "glu_bwd", "rmsnorm_rows", "glu_linear", "rmsnorm_linear", "rmsnorm",
           "rmsnorm_rope", "add_rmsnorm_rows",
           "available", "_target_exp"]
