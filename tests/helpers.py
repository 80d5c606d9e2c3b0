"""Shared tolerances and input builders for the parity tests."""
import math

import torch


def bf16_ulp(v: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 at |v|: 2^(floor(log2|v|) - 7), floored at the smallest normal spacing."""
    a = v.double().abs().clamp_min(2.0 ** -126)
    return torch.ldexp(torch.ones_like(a), (torch.floor(torch.log2(a)) - 7).to(torch.int32))


def gemm_tolerance(ref: torch.Tensor, absprod: torch.Tensor, K: int) -> torch.Tensor:
    """Elementwise bound for a GEMM output against the oracle: one bf16 ulp of the oracle's value
    (the final rounding) plus 8 * sqrt(K) * 2^-24 of sum_k |a_k b_k| (fp32 accumulation in a different
    order from the oracle's fp64 sum, scaled by the epilogue factors already folded into absprod)."""
    return bf16_ulp(ref) + 8.0 * math.sqrt(max(K, 1)) * 2.0 ** -24 * absprod.double()


def assert_close_ulp(y, ref, tol, frac_exact=0.95, what=""):
    y, ref = y.detach().cpu(), ref.detach().cpu()
    assert torch.isfinite(y.float()).all() == torch.isfinite(ref.float()).all(), f"{what}: finiteness differs"
    fin = torch.isfinite(ref.double())
    d = (y.double() - ref.double()).abs()
    bad = (d > tol.cpu()) & fin
    assert not bad.any(), f"{what}: {int(bad.sum())} elements outside tolerance, max excess {(d - tol.cpu())[bad].max().item():.3e}"
    exact = (y.view(torch.int16) == ref.view(torch.int16)).double().mean().item()
    assert exact >= frac_exact, f"{what}: only {exact:.3f} of elements bit-equal"


def rel_err(y, ref):
    """||y - ref|| / ||ref|| in fp64, on the GPU when both tensors are there."""
    dev = ref.device if (y.is_cuda and ref.is_cuda) else "cpu"
    y, ref = y.detach().to(dev).double(), ref.detach().to(dev).double()
    return ((y - ref).norm() / ref.norm()).item()


def edge_rows(R, K, seed=0, device="cpu"):
    """bf16 rows covering the exponent rules' edges: zero row, fp32-subnormal-sized values, exact powers
    of two at bin edges, a single huge element, rows near fp16 overflow, NaN and inf entries."""
    g = torch.Generator().manual_seed(seed)
    e = torch.randint(-40, 41, (R, 1), generator=g).float()
    x = torch.randn(R, K, generator=g) * torch.exp2(e)
    if R > 8:
        x[0] = 0.0
        x[1] = 1e-38
        x[2] = torch.exp2(torch.randint(-20, 20, (K,), generator=g).float())
        x[3, :] = 1e-3
        x[3, K // 2] = 3e4
        x[4] = 65504.0
        x[5] = 2.0 ** 15
        x[6, 1] = float("inf")
        x[7, 2] = float("nan")
    return x.bfloat16().to(device)


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality of 16-bit tensors, treating any two NaNs as equal (NaN payloads differ
    between the GPU's conversions and the oracle's)."""
    a, b = a.detach().cpu(), b.detach().cpu()
    if a.shape != b.shape:
        return False
    both_nan = torch.isnan(a.float()) & torch.isnan(b.float())
    return bool(((a.view(torch.int16) == b.view(torch.int16)) | both_nan).all())


def ulp_distance(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Number of bf16 values between a and b (both bf16): the distance of their bit patterns on the
    ordered integer line (negative values mirrored, so -0 and +0 are one point)."""
    def ordered(t):
        v = t.detach().cpu().contiguous().view(torch.int16).int()
        return torch.where(v < 0, -(v & 0x7FFF), v)
    return (ordered(a) - ordered(b)).abs()


def report(name: str, **values):
    """One greppable line per parity measurement (shown with pytest -s)."""
    parts = " ".join(f"{k}={v:.3e}" if isinstance(v, float) else f"{k}={v}" for k, v in values.items())
    print(f"\nPARITY {name} {parts}")
