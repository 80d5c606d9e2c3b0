"""Scaled bf16 convolutions (tbf16.conv, the reference's tbf16/conv.py): the im2col + tcgen05 GEMM path
and the grouped / depthwise kernel against the oracle's restatement (per-sample power-of-two input
scale, prepared weight rows, fp64 accumulation), elementwise within one bf16 ulp plus the fp32
summation bound; every case also within 3e-3 of an fp64 convolution of the dequantized weight, the
reference's own test bar (tests/test_conv.py there), including inputs whose plain fp16 conversion
overflows or underflows. Case list after the reference's test_conv.py."""
import copy
import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from helpers import assert_close_ulp, gemm_tolerance, rel_err
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

CONV = {1: F.conv1d, 2: F.conv2d, 3: F.conv3d}


def _fp64_ref(conv, x):
    w = conv.dequantized_weight().double()
    b = None if conv.bias is None else conv.bias.double()
    if conv.padding_mode != "zeros":
        x = F.pad(x.double(), conv._reversed_padding_repeated_twice, mode=conv.padding_mode)
        return CONV[x.dim() - 2](x, w, b, conv.stride, 0, conv.dilation, conv.groups)
    return CONV[x.dim() - 2](x.double(), w, b, conv.stride, conv.padding, conv.dilation, conv.groups)


def _run(conv, shape, scale=1.0, channels_last=False, seed=0):
    from tbf16.conv import convert_conv
    torch.manual_seed(seed)
    conv = conv.cuda().bfloat16()
    x = (torch.randn(shape, device="cuda") * scale).bfloat16()
    if channels_last:
        x = x.to(memory_format=torch.channels_last if x.dim() == 4 else torch.channels_last_3d)
    tc = convert_conv(copy.deepcopy(conv))
    with torch.no_grad():
        y = tc(x)
    return tc, x, y


CASES = [
    ("conv2d 3x3", lambda: nn.Conv2d(64, 96, 3, padding=1), (2, 64, 40, 56), False),
    ("conv2d 3x3 no bias stride 2", lambda: nn.Conv2d(64, 96, 3, stride=2, padding=1, bias=False), (2, 64, 40, 56), False),
    ("conv2d 3x3 channels_last", lambda: nn.Conv2d(64, 96, 3, padding=1), (2, 64, 40, 56), True),
    ("conv2d depthwise 5x5 channels_last", lambda: nn.Conv2d(96, 96, 5, padding=2, groups=96, bias=False),
     (1, 96, 16, 16), True),
    ("conv2d grouped 1x1", lambda: nn.Conv2d(96, 96, 1, groups=6, bias=False), (1, 96, 16, 16), False),
    ("conv1d k=4", lambda: nn.Conv1d(48, 64, 4, padding=1), (3, 48, 100), False),
    ("conv3d 3x3x3", lambda: nn.Conv3d(32, 48, 3, padding=1), (1, 32, 5, 24, 40), False),
    ("conv3d 3x3x3 channels_last_3d", lambda: nn.Conv3d(32, 48, 3, padding=1), (1, 32, 5, 24, 40), True),
    ("conv2d rgb in 3x3 (K = 27)", lambda: nn.Conv2d(3, 64, 3, padding=1), (2, 3, 32, 32), False),
    ("conv2d to rgb (O = 3)", lambda: nn.Conv2d(64, 3, 3, padding=1), (2, 64, 32, 32), False),
    ("conv2d 3x3 dilation 2", lambda: nn.Conv2d(32, 40, 3, padding=2, dilation=2), (1, 32, 30, 30), False),
]


@pytest.mark.parametrize("name,make,shape,cl", CASES, ids=[c[0] for c in CASES])
def test_conv_vs_oracle(name, make, shape, cl):
    tc, x, y = _run(make(), shape, channels_last=cl)
    assert y.dtype == torch.bfloat16 and torch.isfinite(y.float()).all()
    y_ref, absacc = orc.conv_scaled(x.contiguous(), tc.weight16, tc.weight_scale, tc.bias, tc.stride, tc.padding,
                                    tc.dilation, tc.groups, tc._tbf16_target_exp)
    assert y.shape == y_ref.shape
    K = tc.weight16[0].numel()
    assert_close_ulp(y.contiguous(), y_ref, gemm_tolerance(y_ref, absacc, K), what=name)
    assert rel_err(y, _fp64_ref(tc, x)) < 3e-3


@pytest.mark.parametrize("scale", [3e4, 1e6, 1e-8])
@pytest.mark.parametrize("nd", [2, 3])
def test_conv_scales(scale, nd):
    """Inputs that overflow (or vanish in) plain fp16 stay accurate: the per-sample scale moves them."""
    make = (lambda: nn.Conv2d(64, 96, 3, padding=1)) if nd == 2 else (lambda: nn.Conv3d(32, 48, 3, padding=1))
    shape = (2, 64, 40, 56) if nd == 2 else (1, 32, 5, 24, 40)
    tc, x, y = _run(make(), shape, scale=scale)
    assert torch.isfinite(y.float()).all()
    assert rel_err(y, _fp64_ref(tc, x)) < 3e-3


def test_conv_pointwise_and_padding_modes():
    """1x1 convolutions take scaled_linear (per-pixel scales, as the reference); reflect padding is
    applied before the zero-padded kernel; padding="same"; a zero sample gives exactly the bias."""
    for make, shape, cl in [(lambda: nn.Conv2d(128, 320, 1), (2, 128, 24, 24), False),
                            (lambda: nn.Conv2d(128, 320, 1), (2, 128, 24, 24), True),
                            (lambda: nn.Conv2d(32, 32, 3, padding=1, padding_mode="reflect"), (1, 32, 33, 47), False),
                            (lambda: nn.Conv2d(16, 24, 4, padding="same"), (2, 16, 20, 21), False)]:
        tc, x, y = _run(make(), shape, channels_last=cl)
        assert y.shape == _fp64_ref(tc, x).shape
        assert rel_err(y, _fp64_ref(tc, x)) < 3e-3
    from tbf16.conv import convert_conv
    conv = convert_conv(nn.Conv2d(8, 16, 3, padding=1).cuda().bfloat16())
    x = torch.zeros(2, 8, 6, 6, device="cuda", dtype=torch.bfloat16)
    x[1] = 1.0
    with torch.no_grad():
        y = conv(x)
    assert torch.equal(y[0], conv.bias.view(16, 1, 1).expand(16, 6, 6))


def test_convert_reaches_nested_and_subclassed_convs():
    import tbf16

    class CausalConv3d(nn.Conv3d):  # own forward, then super().forward (as diffusers' causal convs)
        def __init__(self, *a, **k):
            super().__init__(*a, **k)
            self._pad = (1, 1, 1, 1, 2, 0)
            self.padding = (0, 0, 0)

        def forward(self, x):
            return super().forward(F.pad(x, self._pad))

    model = nn.Sequential(nn.Conv2d(16, 32, 3, padding=1), nn.Sequential(nn.SiLU(), nn.Conv2d(32, 16, 1))).cuda().bfloat16()
    x = torch.randn(1, 16, 20, 20, device="cuda").bfloat16()
    with torch.no_grad():
        r = copy.deepcopy(model).double()(x.double())
        tbf16.convert(model, sdpa=False, force=True)
        y = model(x)
    assert type(model[0]).__name__ == "TBF16Conv2d" and type(model[1][1]).__name__ == "TBF16Conv2d"
    assert rel_err(y, r) < 1e-2
    wrapped = nn.Sequential(CausalConv3d(8, 8, 3)).cuda().bfloat16()
    x3 = torch.randn(1, 8, 4, 10, 10, device="cuda").bfloat16()
    with torch.no_grad():
        r3 = copy.deepcopy(wrapped).double()(x3.double())
        tbf16.convert(wrapped, sdpa=False, force=True)
        assert type(wrapped[0]).__name__ == "TBF16CausalConv3d"
        assert rel_err(wrapped(x3), r3) < 3e-3


# Stride-1 convolutions with C % 64 == 0 and output rows that tile into 128-position boxes take the
# implicit GEMM (TMA loads of each tap's block straight from the scaled channels-last copy): output
# widths below, at and above 128, dilation, valid padding, 3-D, 192 channels (three 64-channel blocks per
# tap), 25 taps, and a pair tile whose second half lies past the last sample (M = 384).
IMPLICIT = [
    ("2d 3x3 Wo=64", lambda: nn.Conv2d(64, 96, 3, padding=1), (2, 64, 32, 64), False),
    ("2d 3x3 Wo=256 channels_last", lambda: nn.Conv2d(128, 128, 3, padding=1), (1, 128, 16, 256), True),
    ("2d 3x3 dilation 2", lambda: nn.Conv2d(64, 64, 3, padding=2, dilation=2, bias=False), (1, 64, 32, 32), False),
    ("2d 3x3 valid", lambda: nn.Conv2d(64, 72, 3), (1, 64, 34, 34), False),
    ("2d 5x5 C=192", lambda: nn.Conv2d(192, 64, 5, padding=2), (2, 192, 16, 16), False),
    ("2d 3x3 M=384", lambda: nn.Conv2d(64, 64, 3, padding=1), (3, 64, 8, 16), False),
    ("3d 3x3x3", lambda: nn.Conv3d(64, 64, 3, padding=1), (1, 64, 4, 16, 32), False),
]


@pytest.mark.parametrize("name,make,shape,cl", IMPLICIT, ids=[c[0] for c in IMPLICIT])
def test_conv_implicit_vs_oracle(name, make, shape, cl):
    from tbf16 import _ext
    from tbf16.conv import scaled_conv
    tc, x, y = _run(make(), shape, channels_last=cl)
    nd = x.dim() - 2
    # the case takes the implicit GEMM
    k = (1,) * (3 - nd) + tuple(tc.weight16.shape[2:])
    xs = x.reshape((x.shape[0], x.shape[1]) + (1,) * (3 - nd) + tuple(x.shape[2:]))
    pad = (0,) * (3 - nd) + tuple(tc.padding)
    dil = (1,) * (3 - nd) + tuple(tc.dilation)
    out = tuple((n + 2 * p - d * (kk - 1) - 1) + 1 for n, p, d, kk in zip(xs.shape[2:], pad, dil, k))
    geom = torch.tensor([*xs.shape, *xs.stride(), *k, 1, 1, 1, *pad, *dil, *out], dtype=torch.int64)
    assert _ext.lib().tbf16_conv_implicit_supported(_ext.ptr(geom), tc.out_channels) == 0
    y_ref, absacc = orc.conv_scaled(x.contiguous(), tc.weight16, tc.weight_scale, tc.bias, tc.stride, tc.padding,
                                    tc.dilation, tc.groups, tc._tbf16_target_exp)
    assert y.shape == y_ref.shape
    K = tc.weight16[0].numel()
    tol = gemm_tolerance(y_ref, absacc, K)
    assert_close_ulp(y.contiguous(), y_ref, tol, what=name)
    assert rel_err(y, _fp64_ref(tc, x)) < 3e-3
    # the im2col path: the same products, so the same result within the fp32 summation bound
    with torch.no_grad():
        y2 = scaled_conv(x, tc.weight16, tc.weight_scale, tc.bias, tc.stride, tc.padding, tc.dilation, tc.groups,
                         tc._tbf16_target_exp, implicit=False)
    assert_close_ulp(y.contiguous(), y2.contiguous().cpu(), 2 * tol, what=name + " vs im2col")


def test_conv_implicit_scales():
    """Samples of very different magnitude in one batch keep their own scale through the implicit GEMM."""
    tc, x, y = _run(nn.Conv2d(64, 64, 3, padding=1), (2, 64, 16, 32))
    x2 = x.clone()
    x2[0] *= 2.0 ** 40
    x2[1] *= 2.0 ** -40
    with torch.no_grad():
        y2 = tc(x2)
    assert torch.isfinite(y2.float()).all()
    r = _fp64_ref(tc, x2)
    for b in range(2):
        assert rel_err(y2[b], r[b]) < 3e-3
