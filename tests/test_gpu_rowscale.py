"""Parity of the HBM-bound scale kernels with the oracle (bit-exact integer exponents and fp16
operands), called through the C ABI. Edge rows: zero, subnormal-sized, exact powers of two, single
outlier, fp16 overflow, inf and NaN entries."""
import math

import pytest
import torch

from helpers import bits_equal, edge_rows
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _ext():
    from tbf16 import _ext
    return _ext


@pytest.mark.parametrize("R,K", [(64, 64), (37, 1032), (8, 20000), (300, 4096), (1, 8), (16, 8192), (5, 16384),
                                 (1024, 2056), (1025, 2056)])
@pytest.mark.parametrize("l1", [False, True])
def test_row_scale_fused(R, K, l1):
    E = _ext()
    x = edge_rows(R, K, seed=R + K).cuda()
    s_inv = torch.empty(R, device="cuda")
    e8 = torch.empty(R, device="cuda", dtype=torch.int8)
    y16 = torch.empty(R, K, device="cuda", dtype=torch.float16)
    E.call("tbf16_row_scale", E.ptr(x), R, K, x.stride(0), 15, int(l1), E.ptr(s_inv), E.ptr(e8), E.ptr(y16), K,
           E.stream_ptr())
    ref = orc.row_scale_fused(x.cpu(), 15, l1)
    # both sides sum L1 norms (near) exactly (fp64 on the GPU, binary128 in the oracle): all rows compare
    assert torch.equal(s_inv.cpu(), ref)
    assert torch.equal(e8.cpu().int(), -torch.log2(ref.double()).round().int())
    # the materialised operand is fp16_rn(x * s) with the same s (gemm_sm75.cu:108,132)
    s = torch.ldexp(torch.ones(R, dtype=torch.float64), -torch.log2(ref.double()).round().int())
    assert bits_equal(y16, orc.f16_rn((x.cpu().double() * s[:, None]).float()))
    s2 = torch.empty(R, device="cuda")
    E.call("tbf16_row_scale", E.ptr(x), R, K, x.stride(0), 15, int(l1), E.ptr(s2), None, None, 0, E.stream_ptr())
    assert torch.equal(s2, s_inv)


@pytest.mark.parametrize("R,K", [(64, 64), (37, 1032), (8, 20000), (257, 4096), (16, 8192), (3, 16384)])
@pytest.mark.parametrize("t", [0, -1, 15])
@pytest.mark.parametrize("l1", [False, True])
def test_quantize_rows(R, K, t, l1):
    from tbf16 import ops
    x = edge_rows(R, K, seed=3 * R + K).cuda()
    y, s = ops.quantize_rows(x, t, l1)
    y_ref, s_ref = orc.quantize_rows(x.cpu(), t, l1)
    assert torch.equal(s.cpu(), s_ref)
    assert bits_equal(y, y_ref)


def test_quantize_rows_strided_input():
    from tbf16 import ops
    big = edge_rows(40, 256, seed=9).cuda()
    x = big[:, 64:192]  # row stride 256, 16-byte aligned start
    y, s = ops.quantize_rows(x, 0, False)
    y_ref, s_ref = orc.quantize_rows(x.cpu().contiguous(), 0, False)
    assert torch.equal(s.cpu(), s_ref) and bits_equal(y, y_ref)


@pytest.mark.parametrize("R,K", [(48, 64), (333, 520), (2048, 256), (0, 64)])
@pytest.mark.parametrize("t", [0, -3])
@pytest.mark.parametrize("with_row_mul", [False, True])
def test_quantize_cols(R, K, t, with_row_mul):
    E = _ext()
    x = edge_rows(R, K, seed=R + 7 * K).cuda() if R else torch.empty(0, K, dtype=torch.bfloat16, device="cuda")
    x = torch.nan_to_num(x.float(), nan=0.0, posinf=1e30).bfloat16()  # keep columns finite for the row_mul fold
    rm = torch.exp2(torch.randint(-8, 9, (R,), generator=torch.Generator().manual_seed(1)).float()).cuda() if with_row_mul else None
    y = torch.empty(R, K, device="cuda", dtype=torch.float16)
    s = torch.empty(K, device="cuda")
    ws = torch.empty(K, device="cuda")
    E.call("tbf16_quantize_cols", E.ptr(x), R, K, x.stride(0) if R else K, t, E.ptr(rm), E.ptr(y), K, E.ptr(s), E.ptr(ws),
           E.stream_ptr())
    y_ref, s_ref = orc.quantize_cols(x.cpu(), t, None if rm is None else rm.cpu())
    assert torch.equal(s.cpu(), s_ref)
    assert bits_equal(y, y_ref)


def _strided_bhsd(B, H, S, D, seed, dtype=torch.bfloat16, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    e = torch.randint(-6, 7, (1, H, 1, 1), generator=g).float()
    t = (torch.randn(B, S, H, D, generator=g) * torch.exp2(e.permute(0, 2, 1, 3)) * scale).to(dtype)
    return t.cuda().permute(0, 2, 1, 3)  # (B, H, S, D) view with strides of (B, S, H, D)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_head_amax_exp_scale_cast(dtype):
    E = _ext()
    B, H, S, D = 2, 6, 300, 64
    x = _strided_bhsd(B, H, S, D, 5, dtype)
    x[1, 2] = 0  # an all-zero head -> exponent 0
    code = E.F16 if dtype == torch.float16 else E.BF16
    amax = torch.empty(B * H, device="cuda")
    e = torch.empty(B * H, device="cuda", dtype=torch.int32)
    E.call("tbf16_head_exp", E.ptr(x), code, B, H, S, D, *x.stride()[:3], E.ptr(e), E.ptr(amax), E.stream_ptr())
    assert torch.equal(amax.cpu().view(B, H), orc.head_amax(x.cpu()))
    assert torch.equal(e.cpu().view(B, H), orc.head_exp(x.cpu()))
    ex = (torch.arange(B * H, dtype=torch.int32) - 5).view(B, H).cuda()
    for out_dtype, out_code in ((torch.float16, E.F16), (torch.bfloat16, E.BF16)):
        y = torch.empty(B, H, S, D, device="cuda", dtype=out_dtype)
        E.call("tbf16_head_scale_cast", E.ptr(x), code, B, H, S, D, *x.stride()[:3], E.ptr(ex), H, 1, E.ptr(y), out_code,
               E.stream_ptr())
        ref = orc.head_scale(x.cpu(), ex.cpu(), out_dtype)
        assert bits_equal(y, ref)


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,D,v_exp", [(1, 4, 4, 128, 128, 64, 13), (2, 8, 2, 96, 200, 128, 0),
                                                     (1, 2, 1, 33, 65, 256, 13)])
def test_prepare_qkv(B, Hq, Hkv, Sq, Sk, D, v_exp):
    E = _ext()
    q = _strided_bhsd(B, Hq, Sq, D, 11, scale=2.0 ** 9)
    k = _strided_bhsd(B, Hkv, Sk, D, 12, scale=2.0 ** -3)
    v = _strided_bhsd(B, Hkv, Sk, D, 13, scale=2.0 ** 5)
    q16 = torch.empty(B, Hq, Sq, D, device="cuda", dtype=torch.float16)
    k16 = torch.empty(B, Hkv, Sk, D, device="cuda", dtype=torch.float16)
    v16 = torch.empty_like(k16)
    a = torch.empty(1, device="cuda", dtype=torch.int32)
    ev = torch.empty(B * Hkv, device="cuda", dtype=torch.int32)
    ws = torch.empty(B * Hq + 2 * B * Hkv, device="cuda")
    E.call("tbf16_prepare_qkv", E.ptr(q), *q.stride()[:3], E.ptr(k), *k.stride()[:3], E.ptr(v), *v.stride()[:3], B, Hq, Hkv,
           Sq, Sk, D, v_exp, E.ptr(q16), E.ptr(k16), E.ptr(v16), E.ptr(a), E.ptr(ev), E.ptr(ws), E.stream_ptr())
    rq, rk, rv, ra, rev = orc.prepare_qkv(q.cpu(), k.cpu(), v.cpu(), v_exp)
    assert int(a.item()) == int(ra)
    assert torch.equal(ev.cpu().view(B, Hkv), rev)
    for got, ref in ((q16, rq), (k16, rk), (v16, rv)):
        assert bits_equal(got, ref)


def test_status_codes():
    E = _ext()
    x = torch.zeros(4, 12, device="cuda", dtype=torch.bfloat16)  # K = 12 is not a multiple of 8
    s = torch.empty(4, device="cuda")
    st = E.lib().tbf16_row_scale(E.ptr(x), 4, 12, 12, 15, 0, E.ptr(s), None, None, 0, E.stream_ptr())
    assert st == 2  # TBF16_ERR_ALIGN
    st = E.lib().tbf16_row_scale(E.ptr(x), -1, 8, 8, 15, 0, E.ptr(s), None, None, 0, E.stream_ptr())
    assert st == 1  # TBF16_ERR_INVALID
    assert E.device_status() == 0
