"""Config 5's model on the scaled path, checked against fp64: Gemma-3-4B-shaped decoder layers (hidden
2560, 8 query / 4 KV heads of 256, GeGLU 10240, RMSNorm before and after each block, QK-norm, RoPE) with
random N(0, 0.02^2) weights, the benchmark's own layer code (bench._GemmaLayer), and residual-stream
outlier channels at ~1e5 so that a plain .half() of the activations overflows. Two layers, 512 tokens.

The same layers run three ways on the same inputs: converted by tbf16.convert (every linear on the
scaled GEMM, attention on the scaled kernel), then also with the producer fusions the benchmark times
(fused norms, GeGLU and RoPE), and natively in bf16 (torch's cuBLAS / SDPA), each against an fp64 copy.
The scaled path must stay finite and be as close to fp64 as native bf16 is (the reference's claim: the
scaled fp16 path matches bf16's accuracy, README.md:102 there)."""
import copy
import math

import pytest
import torch

from helpers import rel_err, report

pytestmark = pytest.mark.gpu


def _rope(seq, dev):
    pos = torch.arange(seq, device=dev, dtype=torch.float32)
    inv = 1.0 / (1e6 ** (torch.arange(0, 256, 2, device=dev, dtype=torch.float32) / 256))
    ang = torch.outer(pos, inv)
    cos = torch.cat([ang.cos(), ang.cos()], -1).bfloat16()[None, None]
    sin = torch.cat([ang.sin(), ang.sin()], -1).bfloat16()[None, None]
    return cos, sin


def test_gemma_layers_vs_fp64_with_fp16_overflowing_residuals():
    import bench
    import tbf16
    dev = torch.device("cuda")
    torch.manual_seed(0)
    seq, hidden, n_layers = 512, 2560, 2
    with torch.device(dev):
        layers = torch.nn.ModuleList([bench._GemmaLayer() for _ in range(n_layers)]).bfloat16()
        for m in layers.modules():
            if isinstance(m, torch.nn.Linear):
                torch.nn.init.normal_(m.weight, std=0.02)
            if isinstance(m, bench._RMSNorm):
                torch.nn.init.normal_(m.weight, std=0.1)
    x0 = (torch.randn(1, seq, hidden, device=dev) * (hidden ** 0.5) * 0.02).bfloat16()
    outlier = torch.zeros(hidden, device=dev, dtype=torch.bfloat16)
    outlier[torch.randperm(hidden, device=dev)[:4]] = 1.0
    x0 = x0 + outlier * 1e5
    assert not torch.isfinite(x0.half()).all()  # the activations do overflow plain fp16
    cos, sin = _rope(seq, dev)

    ref = copy.deepcopy(layers).double()
    native = copy.deepcopy(layers)
    with torch.no_grad():
        x64 = x0.double()
        for layer in ref:
            x64 = layer(x64, cos.double(), sin.double())
        xn = x0
        for layer in native:
            xn = layer(xn, cos, sin)
        tbf16.convert(layers)
        assert isinstance(layers[0].q_proj, tbf16.Linear) and isinstance(layers[1].down_proj, tbf16.Linear)
        try:
            xs = x0
            for layer in layers:
                xs = layer(xs, cos, sin)
            for layer in layers:
                layer.fuse_projections()
            xf = x0
            for layer in layers:
                xf = layer(xf, cos, sin)
        finally:
            tbf16.uninstall_sdpa()
    # what the layers added to the residual stream (the input's own bf16 rounding is common to all paths),
    # over the non-outlier channels (the ~1e5 outliers pass through the residual adds unchanged)
    keep = outlier == 0
    d64 = (x64 - x0.double())[..., keep]
    outs = {"scaled": xs, "scaled_fused": xf, "native_bf16": xn}
    errs = {k: rel_err((v.double() - x0.double())[..., keep], d64) for k, v in outs.items()}
    report("gemma layers vs fp64 (layer outputs, non-outlier channels)", **errs,
           scaled_vs_native=rel_err(xs[..., keep], xn[..., keep]))
    for t in (xs, xf):
        assert torch.isfinite(t.float()).all()
    assert rel_err(xs[..., keep], xn[..., keep]) > 0  # the scaled path really ran (its rounding differs)
    for k in ("scaled", "scaled_fused"):
        assert errs[k] <= 1.25 * errs["native_bf16"] + 1e-3, (k, errs)
