"""Pins the oracle against golden vectors produced by running the reference's own code on CPU
(tests/golden/make_golden.py: the reference's Triton kernels under TRITON_INTERPRET=1 and its torch
fallbacks). Rows or columns where the reference's Triton / torch fallback formulas deliberately differ
from its CUDA formulas (all-zero rows, where the CUDA code clamps) are excluded here and covered
by tests/test_oracle_kat.py."""
import math

import numpy as np
import pytest
import torch

import inputs


def from_u16(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype)


def rows_case(seed, R, K):
    g = torch.Generator().manual_seed(seed)
    e = torch.randint(-30, 31, (R, 1), generator=g).float()
    x = torch.randn(R, K, generator=g) * torch.exp2(e)
    x[0] = 0.0
    x[1, :] = 1e-3
    x[1, 3] = 3e4
    x[2] = torch.exp2(torch.randint(-20, 20, (K,), generator=g).float())
    return x.bfloat16()


def near_pow2(v: torch.Tensor, K: int) -> torch.Tensor:
    """True where an fp32 sum of K terms could round across a power of two."""
    v = v.double().abs().clamp_min(1e-300)
    frac = torch.log2(v) - torch.round(torch.log2(v))
    return frac.abs() < K * 2.0 ** -24 / math.log(2) + 1e-12


@pytest.mark.parametrize("i", [0, 1, 2])
def test_quantize_rows_vs_reference_triton(orc, golden, i):
    seed, R, K = (int(v) for v in golden[f"qr{i}_meta"])
    x = rows_case(seed, R, K)
    assert inputs.checksum(x) == str(golden[f"qr{i}_xsum"])
    for t in (0, -1, 15):
        for l1 in (False, True):
            y_ref = from_u16(golden[f"qr{i}_t{t}_l{int(l1)}_y"], torch.float16)
            s_ref = torch.from_numpy(golden[f"qr{i}_t{t}_l{int(l1)}_s"])
            y, s = orc.quantize_rows(x, t, l1)
            red = orc.row_reduce(x, l1)
            keep = red > 0                                   # zero rows: CUDA clamp differs from Triton
            if l1:
                keep &= ~near_pow2(red, K)                   # fp32 summation order may flip these
            assert keep.sum() >= R - 2
            assert torch.equal(s[keep], s_ref[keep]), (t, l1)
            assert torch.equal(y[keep].view(torch.int16), y_ref[keep].view(torch.int16)), (t, l1)


def test_prepare_weight_vs_reference(orc, golden):
    w = inputs.gemm_w(96, 1024, seed=7)
    assert inputs.checksum(w) == str(golden["pw_xsum"])
    w16, ws = orc.prepare_weight(w)
    assert torch.equal(w16.view(torch.int16), from_u16(golden["pw_w16"], torch.int16))
    assert torch.equal(ws, torch.from_numpy(golden["pw_ws"]))


def _ulp_close(y, ref, scale_bound, frac_exact=0.99):
    """|y - ref| <= 1 bf16 ulp of ref + 2^-10 * scale_bound elementwise (the fp16 rounding of the
    reference's GEMM output can move cancelling sums), and most elements bit-equal.

    The reference's epilogue here ran as a Triton kernel under TRITON_INTERPRET=1, whose numpy cast
    truncates fp32 to bf16 (a GPU rounds to nearest); the pins compare against the oracle with the
    same truncation (oracle.linear_small_m_ref(..., rounding="trunc"))."""
    d = (y.double() - ref.double()).abs()
    from oracle.oracle import bf16_ulp
    assert (d <= bf16_ulp(ref) + 2.0 ** -10 * scale_bound).all()
    assert (y.view(torch.int16) == ref.view(torch.int16)).double().mean() >= frac_exact


@pytest.mark.parametrize("i", [0, 1, 2])
def test_small_m_linear_vs_reference(orc, golden, i):
    M, K, N, sx, sw, sb = (int(v) for v in golden[f"sl{i}_meta"])
    x, w = inputs.gemm_x(M, K, seed=sx), inputs.gemm_w(N, K, seed=sw)
    b = (torch.randn(N, generator=torch.Generator().manual_seed(sb)) * 0.1).bfloat16()
    assert inputs.checksum(x, w, b) == str(golden[f"sl{i}_xsum"])
    w16, ws = orc.prepare_weight(w)
    y = orc.linear_small_m_ref(x, w16, ws, b, rounding="trunc")
    y_ref = from_u16(golden[f"sl{i}_y"], torch.bfloat16)
    bound = (x.double().abs() @ w.double().abs().t())
    _ulp_close(y, y_ref, bound)


def test_config1_vs_reference(orc, golden):
    x, w, b = inputs.config1()
    assert inputs.checksum(x, w, b) == str(golden["c1_xsum"])
    w16, ws = orc.prepare_weight(w)
    assert inputs.checksum(w16) == str(golden["c1_w16sum"])
    assert torch.equal(ws, torch.from_numpy(golden["c1_ws"]))
    y_ref = from_u16(golden["c1_y"], torch.bfloat16)
    bound = (x.double().abs() @ w.double().abs().t())
    _ulp_close(orc.linear_small_m_ref(x, w16, ws, b, rounding="trunc"), y_ref, bound)
    # this build's semantics (fused path: max rows at t=15, no fp16 rounding of the product)
    y, _ = orc.linear_fused(x, w16, ws, b)
    exact = x.double() @ w.double().t() + b.double()
    assert orc.rel_err(y, exact) < 2e-3
    d = (y.double() - orc.linear_small_m_ref(x, w16, ws, b).double()).abs()
    from oracle.oracle import bf16_ulp
    assert (d <= bf16_ulp(exact) + 2.0 ** -10 * bound).all()


@pytest.mark.parametrize("t", [0, -3])
def test_quantize_cols_vs_reference(orc, golden, t):
    x = rows_case(200, 48, 64)
    rm = torch.exp2(torch.randint(-8, 9, (48,), generator=torch.Generator().manual_seed(201)).float())
    assert inputs.checksum(x, rm) == str(golden["qc_xsum"])
    for key, row_mul in ((f"qc_t{t}", None), (f"qcm_t{t}", rm)):
        y, s = orc.quantize_cols(x, t, row_mul)
        assert torch.equal(s, torch.from_numpy(golden[f"{key}_s"]))
        assert torch.equal(y.view(torch.int16), from_u16(golden[f"{key}_y"], torch.int16))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_attention_helpers_vs_reference(orc, golden, i):
    B, H, S, D, Hkv, causal, qk, seed = (int(v) for v in golden[f"at{i}_meta"])
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=seed, Hkv=Hkv, qk_exp=qk)
    assert inputs.checksum(q, k, v) == str(golden[f"at{i}_xsum"])
    assert torch.equal(orc.head_amax(q), torch.from_numpy(golden[f"at{i}_amax_q"]))
    assert torch.equal(orc.head_exp(q), torch.from_numpy(golden[f"at{i}_eq"]))
    for v_exp in (0, 13):
        q16, k16, v16, a, ev = orc.prepare_qkv(q, k, v, v_exp)
        assert int(a) == int(golden[f"at{i}_v{v_exp}_a"])
        assert torch.equal(ev, torch.from_numpy(golden[f"at{i}_v{v_exp}_ev"]))
        for name, t in (("q16", q16), ("k16", k16), ("v16", v16)):
            assert torch.equal(t.view(torch.int16), from_u16(golden[f"at{i}_v{v_exp}_{name}"], torch.int16)), name
    e = torch.arange(B * H, dtype=torch.int32).view(B, H) - 3
    assert torch.equal(orc.head_scale(q, e, torch.float16).view(torch.int16), from_u16(golden[f"at{i}_hs"], torch.int16))


@pytest.mark.parametrize("i", [0, 1, 2])
def test_sdpa_vs_reference(orc, golden, i):
    B, H, S, D, Hkv, causal, qk, seed = (int(v) for v in golden[f"at{i}_meta"])
    q, k, v = inputs.attention_qkv(B, H, S, D, seed=seed, Hkv=Hkv, qk_exp=qk)
    f = orc.sdpa_fwd(q, k, v, is_causal=bool(causal), v_exp=13)
    ref = from_u16(golden[f"at{i}_out"], torch.bfloat16)
    vmax = orc._expand_kv(v.abs().amax(dim=(-2, -1), keepdim=True).double(), H)
    d = (f["out_ref"].double() - ref.double()).abs()
    from oracle.oracle import bf16_ulp
    # CPU fp16 SDPA rounds P and accumulates in its own order: 1 ulp plus 2^-9 of the head's V scale
    assert (d <= bf16_ulp(ref) + 2.0 ** -9 * vmax).all()
    exact = orc.sdpa_fwd(q, k, v, is_causal=bool(causal), v_exp=13)["o16"]
    assert orc.rel_err(f["out"], exact * torch.ldexp(torch.ones(()), orc.expand_heads(f["ev"], H).double())[..., None, None]) < 4e-3
