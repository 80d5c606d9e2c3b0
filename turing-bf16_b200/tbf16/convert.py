"""In-place conversion of a bf16 model onto this build's sm_100a kernels (the reference's tbf16.convert).

    tbf16.convert(model)               # inference: weights stored as fp16 rows + power-of-two scales
    tbf16.convert(pipe)                # a pipeline object: each nn.Module in pipe.components
    tbf16.convert(model, train=True)   # training / fine-tuning: forward and backward on the kernels

The conversion is a plan over the module tree, made before anything changes, then applied:

  inference  every bf16 CUDA nn.Linear whose weight no other module shares becomes a `Linear` that keeps
             only `weight16` (fp16 [N, K]) and `weight_scale` (fp32 [N], inverse power-of-two row
             scales) -- the reference's buffer format, so the memory is the bf16 weight's; bf16
             Conv1d/2d/3d are converted in place by tbf16.conv when conv=True.
  training   every nn.Linear is re-classed as `TrainLinear` (parameters, hooks and PEFT wrappers stay
             as they are); its bf16 CUDA calls run through tbf16.autograd.

Both install a hook on F.scaled_dot_product_attention that sends eligible bf16 calls to the scaled
attention (`attention_route`). The same routing decisions serve `tbf16.patch()`.
"""
import collections
import os
import warnings

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import autograd
from .attention import sdpa
from .conv import convert_conv, convertible
from .ops import prepare_weight, scaled_linear

# Training: layers with a dimension below this (LoRA adapters and the like) take fp32 math instead of the
# scaled kernels (the reference's TBF16_MIN_DIM, default 128).
MIN_DIM = int(os.environ.get("TBF16_MIN_DIM", 128))

# Attention calls with fewer query rows (token-by-token decoding) stay on torch's kernel (the reference's
# threshold).
MIN_QUERY_ROWS = 16

# Head dims the scaled attention takes (the kernels zero-pad smaller ones to 64 / 128 / 256), forward and
# backward: up to 256, the reference's limit.
MAX_HEAD_DIM = 256
MAX_HEAD_DIM_TRAIN = 256

_native_sdpa = F.scaled_dot_product_attention


# ----------------------------------------------------------------------------------------------- routing

def _bf16_cuda(*ts) -> bool:
    return all(t.is_cuda and t.dtype == torch.bfloat16 for t in ts)


def _under_bf16_autocast(t) -> bool:
    return t.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16


def _as_autocast_would(*ts):
    """The casts a bf16 autocast region would apply, done here (and differentiably) because the routed
    kernels run with autocast disabled."""
    return tuple(None if t is None else t.to(torch.bfloat16) for t in ts)


def attention_route(q, k, v, min_rows=MIN_QUERY_ROWS) -> str:
    """'scaled', 'scaled_train' or 'native' for an F.scaled_dot_product_attention call on q, k, v:
    bf16 CUDA 4-D tensors with head dim <= MAX_HEAD_DIM and at least min_rows query rows take the scaled
    kernels ('scaled_train' when autograd records, for head dims up to MAX_HEAD_DIM_TRAIN)."""
    if not (_bf16_cuda(q, k, v) and q.dim() == 4 and q.shape[-1] <= MAX_HEAD_DIM and q.shape[-2] >= min_rows):
        return "native"
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        return "scaled_train" if q.shape[-1] <= MAX_HEAD_DIM_TRAIN else "native"
    return "scaled"


def _sdpa(query, key, value, *args, **kwargs):  # torch's parameter names: callers pass them as keywords
    if _under_bf16_autocast(query):
        query, key, value = _as_autocast_would(query, key, value)
    route = attention_route(query, key, value)
    fn = {"scaled": sdpa, "scaled_train": autograd.sdpa}.get(route, _native_sdpa)
    return fn(query, key, value, *args, **kwargs)


def install_sdpa():
    """Route F.scaled_dot_product_attention through `attention_route` (undo with uninstall_sdpa)."""
    F.scaled_dot_product_attention = _sdpa
    torch.nn.functional.scaled_dot_product_attention = _sdpa


def uninstall_sdpa():
    F.scaled_dot_product_attention = _native_sdpa


# ----------------------------------------------------------------------------------------------- layers

def dequantize(w16: torch.Tensor, w_sinv: torch.Tensor) -> torch.Tensor:
    """bf16 weight rows from the stored fp16 rows and their inverse scales (exact: the scales are powers of
    two and every fp16 row value times its scale is a bf16 value)."""
    return (w16.float() * w_sinv.view((-1,) + (1,) * (w16.dim() - 1))).bfloat16()


class Linear(nn.Module):
    """Inference stand-in for a bf16 nn.Linear. Holds `weight16` / `weight_scale` (the reference's storage
    format, convert.py:33-44 there) and `bias`; `weight` is a bf16 view rebuilt on demand for code that
    reads it. bf16 inputs outside autograd take the scaled GEMM; anything else runs F.linear on the
    rebuilt weight."""

    def __init__(self, lin: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = lin.in_features, lin.out_features
        w16, w_sinv = prepare_weight(lin.weight.data)
        self.register_buffer("weight16", w16)
        self.register_buffer("weight_scale", w_sinv)
        self.bias = lin.bias

    @property
    def weight(self):
        return dequantize(self.weight16, self.weight_scale)

    def forward(self, x):
        recording = torch.is_grad_enabled() and x.requires_grad
        if x.dtype == torch.bfloat16 and not recording:
            return scaled_linear(x, self.weight16, self.weight_scale, self.bias)
        bias = None if self.bias is None else self.bias.to(x.dtype)
        return F.linear(x, self.weight.to(x.dtype), bias)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


class TrainLinear(nn.Linear):
    """nn.Linear whose bf16 CUDA calls run on the scaled kernels: autograd.linear when gradients are
    recorded, the inference GEMM on freshly prepared weight rows when not, fp32 math for layers with a
    dimension below MIN_DIM. Installed by re-classing an existing nn.Linear."""

    def forward(self, x):
        w, b = self.weight, self.bias
        if _under_bf16_autocast(x):
            x, w, b = _as_autocast_would(x, w, b)
        if not _bf16_cuda(x, w):
            return F.linear(x, w, b)
        if min(w.shape) < MIN_DIM:
            return autograd.FP32LinearFn.apply(x, w, b)
        if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
            return autograd.linear(x, w, b)
        return scaled_linear(x, *prepare_weight(w), b)


# ----------------------------------------------------------------------------------------------- convert

def is_supported_gpu(device=None) -> bool:
    """True on the GPUs this build's kernels run on: sm_100 (B200)."""
    return torch.cuda.is_available() and torch.cuda.get_device_capability(device) == (10, 0)


def _modules_to_convert(model):
    if isinstance(model, nn.Module):
        return [model]
    components = getattr(model, "components", None)
    if isinstance(components, dict):
        return [c for c in components.values() if isinstance(c, nn.Module)]
    raise TypeError(f"tbf16.convert: expected an nn.Module or a pipeline with a `components` dict, got {type(model)}")


def _shared_parameter_ids(root: nn.Module):
    """ids of parameters registered on more than one module (a tied lm_head and embedding, say): converting
    such a layer would keep a second copy of the weight, so it stays native."""
    owners = collections.Counter(id(p) for m in root.modules() for p in m.parameters(recurse=False))
    return {pid for pid, n in owners.items() if n > 1}


def _inference_plan(root: nn.Module, conv: bool):
    """(parent, attribute name, child, kind) for every layer to convert, collected before any change."""
    shared = _shared_parameter_ids(root)
    plan = []
    for parent in root.modules():
        for name, child in parent.named_children():
            if type(child) is nn.Linear and child.weight.dtype == torch.bfloat16 and child.weight.is_cuda:
                kind = "linear"
            elif conv and convertible(child):
                kind = "conv"
            else:
                continue
            if id(child.weight) not in shared:
                plan.append((parent, name, child, kind))
    return plan


def _convert_for_inference(root: nn.Module, conv: bool):
    for parent, name, child, kind in _inference_plan(root, conv):
        if kind == "linear":
            setattr(parent, name, Linear(child))
            child.weight = None  # release the bf16 weight now rather than when the walk ends
        else:
            convert_conv(child)
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


def _convert_for_training(root: nn.Module):
    for m in root.modules():
        if type(m) is nn.Linear:
            m.__class__ = TrainLinear


def convert(model, train: bool = False, sdpa: bool = True, force: bool = False, conv: bool = True):
    """Convert `model` (an nn.Module, or a pipeline whose `components` dict holds modules) in place and
    return it. On a GPU other than sm_100 this warns and changes nothing unless force=True.
    train: re-class nn.Linear as TrainLinear instead of replacing it. sdpa: install the attention hook.
    conv: also convert bf16 convolutions (inference only)."""
    if not force and not is_supported_gpu():
        warnings.warn("tbf16.convert: this build's kernels need an sm_100 (B200) GPU; the model is left unchanged "
                      "(pass force=True to convert anyway).")
        return model
    for root in _modules_to_convert(model):
        if train:
            _convert_for_training(root)
        else:
            _convert_for_inference(root, conv)
    if sdpa:
        install_sdpa()
    return model
