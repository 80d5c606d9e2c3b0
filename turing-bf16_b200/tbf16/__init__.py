"""tbf16 on B200: bf16 models on fp16 tensor cores with exact power-of-two scales, sm_100a kernels.

Drop-in for tech-cosmos/turing-bf16's public API (tbf16.convert, tbf16.ops, tbf16.attention,
tbf16.autograd, tbf16.patch). The compute runs in libtbf16_sm100.so (hand-written tcgen05 / TMA
kernels) through a C ABI; there is no CPU or library fallback.
"""
__version__ = "0.1.0+b200"

from . import autograd, ops
from .attention import sdpa
from .convert import Linear, TrainLinear, convert, install_sdpa, is_supported_gpu, uninstall_sdpa
from .ops import prepare_weight, quantize_rows, scaled_linear
from .patch import TuringBF16Mode, patch

__all__ = ["quantize_rows", "scaled_linear", "prepare_weight", "sdpa", "patch", "TuringBF16Mode", "convert",
           "Linear", "TrainLinear", "autograd", "install_sdpa", "uninstall_sdpa", "is_supported_gpu"]
