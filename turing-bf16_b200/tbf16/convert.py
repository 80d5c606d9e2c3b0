"""Convert a bf16 model in place so its linear layers and attention run on this build's kernels.

    tbf16.convert(model)               # inference
    tbf16.convert(pipe)                # diffusers-style pipeline: every nn.Module component
    tbf16.convert(model, train=True)   # training / fine-tuning (also after PEFT/LoRA wrapping)

Same API and routing rules as the reference's tbf16/convert.py. Inference: every bf16 nn.Linear
becomes a tbf16.Linear holding its weight as fp16 plus one exact power-of-two scale per output row
(same memory as bf16, same values). Training: every nn.Linear becomes a tbf16.TrainLinear (an
nn.Linear subclass with the same parameters) whose forward and backward run on the scaled kernels.
Both route F.scaled_dot_product_attention to the scaled attention for bf16 inputs.

Differences from the reference: the reference applies only to GPUs without bf16 tensor cores
(Volta/Turing); this build targets B200, so is_supported_gpu() is true on sm_100. With conv=True,
bf16 Conv1d/2d/3d run on the scaled convolutions of tbf16.conv (inference only), as in the reference.
"""
import os
import warnings

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import autograd
from .attention import sdpa
from .conv import convert_conv, convertible
from .ops import prepare_weight, scaled_linear

# Train mode: linear layers with in or out features below this run in fp32 (reference convert.py:27).
MIN_DIM = int(os.environ.get("TBF16_MIN_DIM", 128))

# Attention with fewer query rows (decoding) runs natively (reference convert.py:30).
MIN_QUERY_ROWS = 16

# Head dims the scaled attention kernels take (smaller ones are zero-padded up to 64 / 128 / 256): the
# forward up to 256 (the reference's routing limit), the backward up to 128.
MAX_HEAD_DIM = 256
MAX_HEAD_DIM_TRAIN = 128


class Linear(nn.Module):
    """Inference linear: weight16 (fp16 [N, K]) and weight_scale (fp32 [N]) buffers, as the reference
    stores them (reference convert.py:33-52)."""

    def __init__(self, lin: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = lin.in_features, lin.out_features
        w16, ws = prepare_weight(lin.weight.data)
        self.register_buffer("weight16", w16)
        self.register_buffer("weight_scale", ws)
        self.bias = lin.bias

    @property
    def weight(self):  # bf16 view for code that reads .weight; materialised on demand
        return (self.weight16.float() * self.weight_scale[:, None]).bfloat16()

    def forward(self, x):
        if x.dtype != torch.bfloat16 or torch.is_grad_enabled() and x.requires_grad:
            return F.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))
        return scaled_linear(x, self.weight16, self.weight_scale, self.bias)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


class TrainLinear(nn.Linear):
    """nn.Linear whose bf16 forward and backward run on the scaled kernels. Swapped in by changing
    __class__, so parameters, hooks and PEFT wrappers are untouched (reference convert.py:55-73)."""

    def forward(self, x):
        w, b = self.weight, self.bias
        if x.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
            # bf16 mixed precision (fp32 master weights): do autocast's casts here, differentiably
            x, w = x.to(torch.bfloat16), w.to(torch.bfloat16)
            b = None if b is None else b.to(torch.bfloat16)
        if x.dtype == w.dtype == torch.bfloat16 and x.is_cuda and min(w.shape) < MIN_DIM:
            # skinny layers (e.g. LoRA adapters): fp32 math, as in the reference
            return autograd.FP32LinearFn.apply(x, w, b)
        if x.dtype == w.dtype == torch.bfloat16 and x.is_cuda:
            if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
                return autograd.linear(x, w, b)
            return scaled_linear(x, *prepare_weight(w), b)
        return F.linear(x, w, b)


_native_sdpa = F.scaled_dot_product_attention


def _sdpa(query, key, value, *args, **kwargs):  # torch's parameter names: callers pass them as keywords
    """Routing of F.scaled_dot_product_attention (reference convert.py:79-88): bf16 CUDA 4-D inputs with
    head dim <= MAX_HEAD_DIM and at least MIN_QUERY_ROWS query rows take the scaled path."""
    q, k, v = query, key, value
    if q.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        q, k, v = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)  # what autocast would do
    if (q.dtype == k.dtype == v.dtype == torch.bfloat16 and q.is_cuda and q.dim() == 4
            and q.shape[-1] <= MAX_HEAD_DIM and q.shape[-2] >= MIN_QUERY_ROWS):
        if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
            if q.shape[-1] <= MAX_HEAD_DIM_TRAIN:
                return autograd.sdpa(q, k, v, *args, **kwargs)
            return _native_sdpa(q, k, v, *args, **kwargs)  # no head-dim-256 backward kernel yet
        return sdpa(q, k, v, *args, **kwargs)
    return _native_sdpa(q, k, v, *args, **kwargs)


def install_sdpa():
    F.scaled_dot_product_attention = _sdpa
    torch.nn.functional.scaled_dot_product_attention = _sdpa


def uninstall_sdpa():
    F.scaled_dot_product_attention = _native_sdpa


def is_supported_gpu(device=None) -> bool:
    """True on the GPUs this build's kernels run on: sm_100 (B200)."""
    if not torch.cuda.is_available():
        return False
    return torch.cuda.get_device_capability(device) == (10, 0)


def convert(model, train: bool = False, sdpa: bool = True, force: bool = False, conv: bool = True):
    """Convert in place and return the model (an nn.Module or a pipeline with a `components` dict).
    A no-op (with a warning) on GPUs this build does not target, unless force=True.
    conv: also convert bf16 Conv1d/2d/3d (inference only)."""
    if not force and not is_supported_gpu():
        warnings.warn("tbf16.convert: this build's kernels need an sm_100 (B200) GPU; leaving the model unchanged. "
                      "Pass force=True to convert anyway.")
        return model
    if not isinstance(model, nn.Module) and isinstance(getattr(model, "components", None), dict):
        for c in model.components.values():
            if isinstance(c, nn.Module):
                convert(c, train=train, sdpa=False, force=force, conv=conv)
        if sdpa:
            install_sdpa()
        return model
    if train:
        for mod in model.modules():
            if type(mod) is nn.Linear:
                mod.__class__ = TrainLinear
        if sdpa:
            install_sdpa()
        return model
    # A weight shared with another module (e.g. lm_head tied to the embedding) would be stored twice,
    # so those layers stay native.
    owners = {}
    for mod in model.modules():
        for p in mod.parameters(recurse=False):
            owners[id(p)] = owners.get(id(p), 0) + 1
    for _name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if (type(child) is nn.Linear and child.weight.dtype == torch.bfloat16 and child.weight.is_cuda
                    and owners[id(child.weight)] == 1):
                setattr(mod, cname, Linear(child))
                child.weight = None  # free the bf16 copy now, not when convert() returns
            elif conv and convertible(child) and owners[id(child.weight)] == 1:
                convert_conv(child)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    if sdpa:
        install_sdpa()
    return model
