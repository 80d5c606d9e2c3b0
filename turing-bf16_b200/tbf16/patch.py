"""Run unmodified bf16 PyTorch code on the scaled kernels without converting the model:

    with tbf16.patch():
        out = model(**inputs)

A torch function mode that intercepts two functions on bf16 CUDA tensors while autograd is off:
F.linear (two or more rows: the scaled GEMM, on fp16 weight rows prepared once per weight tensor and
prepared again after the weight changes in place) and F.scaled_dot_product_attention (the routing of
tbf16.convert's attention hook, with the mode's own query-row threshold). Every other call, and every
call it declines, runs unchanged. Counters of taken and declined calls are in `mode.stats`.
"""
import torch
import torch.nn.functional as F
from torch.overrides import TorchFunctionMode
from torch.utils.weak import WeakIdKeyDictionary

from .attention import sdpa
from .convert import _bf16_cuda, attention_route
from .ops import prepare_weight, scaled_linear

# Calls with fewer rows than this stay native: attention query rows (decoding), and F.linear with a
# single row.
MIN_ROWS = 16


class _PreparedWeights:
    """fp16 rows + inverse row scales per weight tensor, keyed by the tensor's identity (entries die with
    it) and invalidated by its version counter (in-place updates)."""

    def __init__(self):
        self._entries = WeakIdKeyDictionary()

    def __call__(self, w):
        entry = self._entries.get(w)
        if entry is None or entry[0] != w._version:
            entry = (w._version, *prepare_weight(w.detach()))
            self._entries[w] = entry
        return entry[1], entry[2]


def _split_sdpa_args(args, kwargs):
    """(q, k, v, remaining positional args, remaining keyword args): q, k and v may arrive as keywords
    (diffusers passes query=, key=, value=)."""
    kwargs = dict(kwargs)
    qkv = [args[i] if i < len(args) else kwargs.pop(name) for i, name in enumerate(("query", "key", "value"))]
    return (*qkv, args[3:], kwargs)


class TuringBF16Mode(TorchFunctionMode):
    def __init__(self, min_rows=MIN_ROWS):
        super().__init__()
        self.min_rows = min_rows
        self._weights = _PreparedWeights()
        self.stats = {"linear": 0, "linear_native": 0, "sdpa": 0, "sdpa_native": 0}

    def _linear(self, func, args, kwargs):
        x, w = args[0], args[1]
        bias = args[2] if len(args) > 2 else kwargs.get("bias")
        if torch.is_grad_enabled() or not _bf16_cuda(x, w):
            return func(*args, **kwargs)
        if x.numel() // max(x.shape[-1], 1) < 2:  # one row: not worth a scaled call
            self.stats["linear_native"] += 1
            return func(*args, **kwargs)
        self.stats["linear"] += 1
        return scaled_linear(x, *self._weights(w), bias)

    def _attention(self, func, args, kwargs):
        q, k, v, rest, kw = _split_sdpa_args(args, kwargs)
        if not torch.is_grad_enabled() and attention_route(q, k, v, self.min_rows) == "scaled":
            self.stats["sdpa"] += 1
            return sdpa(q, k, v, *rest, **kw)
        self.stats["sdpa_native"] += 1
        return func(q, k, v, *rest, **kw)

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func is F.linear:
            return self._linear(func, args, kwargs)
        if func is F.scaled_dot_product_attention:
            return self._attention(func, args, kwargs)
        return func(*args, **kwargs)


def patch(min_rows=MIN_ROWS):
    """Context manager (a TuringBF16Mode). Inference only: with autograd on, calls run natively."""
    return TuringBF16Mode(min_rows)
