"""bf16 convolutions on the B200 kernels with exact power-of-two scales (reference tbf16/conv.py).

Same trick as the linear layers: the weight gets one exact power-of-two scale per output channel, the
input one per sample (a convolution mixes positions, so rows cannot be scaled separately), the products
accumulate in fp32 and the scales are undone in the bf16 epilogue. Same API as the reference module:
convertible(m), convert_conv(conv) (in place, class swap so subclass forwards keep working,
`.weight` becomes None, `.dequantized_weight()` gives it back), and convert(..., conv=True) uses them.

Routing: 1x1 convolutions (stride 1, no padding, one group) are per-pixel linear layers and go through
scaled_linear, as in the reference. Other convolutions with one group run the tcgen05 GEMM against the
weight rows in (taps, channels) order, output channels-last: stride-1 convolutions with channels in
multiples of 64 and output rows that tile into 128-position boxes as an implicit GEMM (the GEMM's TMA
loads each tap's input block from a scaled channels-last fp16 copy, padding as zero fill); the rest
through im2col rows (16-byte tap copies from that copy for channels in multiples of 8, else a generic
im2col). Grouped and depthwise convolutions run a direct kernel.
The reference ends in a cuDNN fp16 convolution whose output is rounded to fp16 before the scales are
applied; here the fp32 sum is scaled and rounded to bf16 once.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from ._ext import call, lib, ptr, require_cuda, stream_ptr
from .ops import _bias_ok, _gemm_f16, _target_exp, prepare_weight, scaled_linear


def _triple(v, nd, fill):
    """Per-dimension values of a conv attribute, as (d, h, w) with `fill` for the dimensions a 1-D or 2-D
    convolution does not have."""
    v = tuple(v) if isinstance(v, (tuple, list)) else (v,) * nd
    return (fill,) * (3 - nd) + v


def _sample_scales(x, t):
    """(e int32 [B], 2^e fp32 [B]) for x bf16 with dense samples."""
    B = x.shape[0]
    n = x[0].numel()
    ld = x.stride(0) if B > 1 else n  # a single sample's batch stride is arbitrary
    amax = torch.empty(B, device=x.device, dtype=torch.float32)
    e = torch.empty(B, device=x.device, dtype=torch.int32)
    scale = torch.empty(B, device=x.device, dtype=torch.float32)
    call("tbf16_conv_sample_scale", ptr(x), B, n, ld, int(t), ptr(amax), ptr(e), ptr(scale),
         stream_ptr(x.device))
    return e, scale


def _dense(x):
    """x itself when each sample is one dense block (contiguous or channels-last), else a contiguous copy."""
    if x.is_contiguous():
        return x
    for fmt in (torch.channels_last, torch.channels_last_3d):
        try:
            if x.is_contiguous(memory_format=fmt):
                return x
        except RuntimeError:
            pass
    return x.contiguous()


def _taps_last(weight16):
    """The weight as [O, taps * C] rows with the channels fastest, for the channels-last im2col."""
    return weight16.movedim(1, -1).reshape(weight16.shape[0], -1).contiguous()


def scaled_conv(x, weight16, weight_scale, bias, stride, padding, dilation, groups, target_exp, wk16=None, wcl16=None,
                implicit=True):
    """The scaled convolution of a bf16 input with a prepared weight (weight16 fp16 [O, C/groups, *k],
    weight_scale fp32 [O]); zero padding only (other padding modes are applied by the caller). wk16: the
    weight as [O, K] rows padded to a multiple of 8; wcl16: as [O, taps * C] rows (channels fastest) for
    C a multiple of 8; each made on the fly when None. implicit=False keeps a convolution the implicit GEMM
    supports on the im2col path (same result up to the fp32 summation order)."""
    require_cuda(x, weight16, weight_scale)
    nd = x.dim() - 2
    x = _dense(x)
    xs = x.reshape((x.shape[0], x.shape[1]) + (1,) * (3 - nd) + tuple(x.shape[2:]))
    B, C, D, H, W = xs.shape
    O = weight16.shape[0]
    k = (1,) * (3 - nd) + tuple(weight16.shape[2:])
    st, pd, dl = _triple(stride, nd, 1), _triple(padding, nd, 0), _triple(dilation, nd, 1)
    out = tuple((n + 2 * p - d * (kk - 1) - 1) // s + 1 for n, p, d, kk, s in zip((D, H, W), pd, dl, k, st))
    if min(out) <= 0:
        raise RuntimeError("tbf16 conv: the kernel does not fit the padded input")
    geom = torch.tensor([B, C, D, H, W, *xs.stride(), *k, *st, *pd, *dl, *out], dtype=torch.int64)
    b = _bias_ok(bias, O, x.device)
    ws = weight_scale.contiguous().float()
    out_shape = (B, O) + tuple(out[3 - nd:])
    M = B * out[0] * out[1] * out[2]
    if groups == 1 and implicit and lib().tbf16_conv_implicit_supported(ptr(geom), O) == 0:
        wk16 = _taps_last(weight16) if wcl16 is None else wcl16
        amax = torch.empty(B, device=x.device, dtype=torch.float32)
        e = torch.empty(B, device=x.device, dtype=torch.int32)
        scale = torch.empty(B, device=x.device, dtype=torch.float32)
        x16cl = torch.empty((B, D, H, W, C), device=x.device, dtype=torch.float16)
        y = torch.empty((M, O), device=x.device, dtype=torch.bfloat16)
        call("tbf16_conv_implicit", ptr(xs), ptr(geom), int(target_exp), ptr(amax), ptr(e), ptr(scale), ptr(x16cl),
             ptr(wk16), O, ptr(ws), ptr(b), ptr(y), stream_ptr(x.device))
        return y.reshape((B,) + tuple(out[3 - nd:]) + (O,)).movedim(-1, 1)
    e, scale = _sample_scales(xs, target_exp)
    if groups == 1:
        K = weight16[0].numel()
        row_scale = torch.empty((M,), device=x.device, dtype=torch.float32)
        if C % 8 == 0:  # channels-last fp16 copy, then 16-byte tap copies (taps x channels columns)
            Kp = K
            wk16 = _taps_last(weight16) if wcl16 is None else wcl16
            x16cl = torch.empty((B, D, H, W, C), device=x.device, dtype=torch.float16)
            cols = torch.empty((M, Kp), device=x.device, dtype=torch.float16)
            call("tbf16_conv_im2col_cl", ptr(xs), ptr(geom), ptr(e), ptr(scale), ptr(x16cl), ptr(cols), ptr(row_scale),
                 stream_ptr(x.device))
        else:
            Kp = (K + 7) // 8 * 8
            if wk16 is None:
                wk16 = weight16.reshape(O, K)
                if Kp != K:
                    wk16 = F.pad(wk16, (0, Kp - K))
            cols = torch.empty((M, Kp), device=x.device, dtype=torch.float16)
            call("tbf16_conv_im2col", ptr(xs), ptr(geom), K, Kp, ptr(e), ptr(scale), ptr(cols), ptr(row_scale),
                 stream_ptr(x.device))
        if O % 8:  # the GEMM writes 16-byte output rows: pad the channels and slice them off
            Op = (O + 7) // 8 * 8
            y = _gemm_f16(cols, 0, F.pad(wk16, (0, 0, 0, Op - O)), 0, M, Op, Kp, row_scale,
                          F.pad(ws, (0, Op - O), value=1.0), None if b is None else F.pad(b, (0, Op - O)))[:, :O]
        else:
            y = _gemm_f16(cols, 0, wk16, 0, M, O, Kp, row_scale, ws, b)
        # [B, Do, Ho, Wo, O] rows -> (B, O, *spatial) with channels-last strides
        y = y.reshape((B,) + tuple(out[3 - nd:]) + (O,))
        return y.movedim(-1, 1)
    y = torch.empty(out_shape, device=x.device, dtype=torch.bfloat16)
    call("tbf16_conv_grouped", ptr(xs), ptr(geom), O, groups, ptr(weight16.contiguous()), ptr(ws), ptr(b), ptr(e),
         ptr(scale), ptr(y), stream_ptr(x.device))
    return y


def _zero_padding(conv, x):
    """(x, padding) with the convolution's padding expressed as zeros around x for scaled_conv: non-zero
    padding modes are applied to x here; "valid" is 0; "same" (stride 1) splits the total padding as
    torch does, an odd total putting its extra element at the end."""
    if conv.padding_mode != "zeros":
        return F.pad(x, conv._reversed_padding_repeated_twice, mode=conv.padding_mode), 0
    if not isinstance(conv.padding, str):
        return x, conv.padding
    if conv.padding == "valid":
        return x, 0
    total = [d * (k - 1) for d, k in zip(conv.dilation, conv.kernel_size)]
    if any(t % 2 for t in total):
        x = F.pad(x, [p for t in reversed(total) for p in (0, t % 2)])
    return x, tuple(t // 2 for t in total)


class _ScaledConv:
    """Mixed in ahead of a bf16 convolution's own class by convert_conv, so that class's forward (and any
    subclass logic around it) still runs and only the innermost `_conv_forward` changes: bf16 inputs
    outside autograd take scaled_conv on the fp16 weight rows; anything else the class's own convolution
    on the rebuilt bf16 weight."""

    def dequantized_weight(self):
        """The bf16 weight rebuilt from `weight16` and `weight_scale` (exact)."""
        scale = self.weight_scale.view((-1,) + (1,) * (self.weight16.dim() - 1))
        return (self.weight16.float() * scale).bfloat16()

    def _conv_forward(self, x, weight, bias):
        # `weight` is the removed bf16 parameter (None): the layer's weight lives in weight16 / weight_scale
        if x.dtype != torch.bfloat16 or (torch.is_grad_enabled() and x.requires_grad):
            b = None if bias is None else bias.to(x.dtype)
            return super()._conv_forward(x, self.dequantized_weight().to(x.dtype), b)
        if self._tbf16_pointwise:  # a per-pixel linear layer
            rows = self.weight16.view(self.out_channels, -1)
            return scaled_linear(x.movedim(1, -1), rows, self.weight_scale, bias).movedim(-1, 1)
        x, padding = _zero_padding(self, x)
        return scaled_conv(x, self.weight16, self.weight_scale, bias, self.stride, padding, self.dilation,
                           self.groups, self._tbf16_target_exp, getattr(self, "_tbf16_wk16", None),
                           getattr(self, "_tbf16_wcl16", None))


_SCALED_CLASSES = {}


def _scaled_class_for(cls):
    """The class a converted `cls` instance takes: _ScaledConv ahead of cls, made once per class."""
    if cls not in _SCALED_CLASSES:
        _SCALED_CLASSES[cls] = type(f"TBF16{cls.__name__}", (_ScaledConv, cls), {})
    return _SCALED_CLASSES[cls]


def convertible(m: nn.Module) -> bool:
    """A Conv1d/2d/3d (or subclass) with a bf16 CUDA weight that has not been converted yet."""
    return (isinstance(m, (nn.Conv1d, nn.Conv2d, nn.Conv3d)) and not isinstance(m, _ScaledConv)
            and isinstance(m.weight, torch.Tensor) and m.weight.dtype == torch.bfloat16 and m.weight.is_cuda)


def _is_pointwise(conv) -> bool:
    unpadded = conv.padding == "valid" or (not isinstance(conv.padding, str) and not any(conv.padding))
    return (conv.groups == 1 and unpadded and all(k == 1 for k in conv.kernel_size)
            and all(s == 1 for s in conv.stride))


def convert_conv(conv: nn.Module):
    """Convert one bf16 convolution in place (reference conv.py:86-103 behaviour): the bf16 weight
    parameter is replaced by `weight16` (fp16, the weight's shape) and `weight_scale` (fp32 [O], inverse
    power-of-two scales of the output channels' rows), plus the GEMM's row layouts of the weight, and the
    instance is re-classed (_scaled_class_for). `.weight` becomes None; `.dequantized_weight()` rebuilds it."""
    w = conv.weight.data
    O, K = w.shape[0], w[0].numel()
    rows16, w_sinv = prepare_weight(w.reshape(O, K))  # [O, K rounded up to a multiple of 8]
    del conv._parameters["weight"]
    conv.register_parameter("weight", None)
    conv.register_buffer("weight16", rows16[:, :K].contiguous().view_as(w))
    conv.register_buffer("weight_scale", w_sinv)
    if conv.groups == 1:
        if w.shape[1] % 8 == 0:  # rows in (taps, channels) order for the channels-last im2col / implicit GEMM
            conv.register_buffer("_tbf16_wcl16", _taps_last(conv.weight16), persistent=False)
        else:  # [O, K] rows padded to a multiple of 8 (a view of weight16 when K already is one)
            conv.register_buffer("_tbf16_wk16", conv.weight16.view(O, K) if K % 8 == 0 else rows16, persistent=False)
    conv._tbf16_target_exp = _target_exp(K)
    conv._tbf16_pointwise = _is_pointwise(conv)
    conv.__class__ = _scaled_class_for(type(conv))
    return conv
