"""tbf16_quantize_cols_noalloc: the column quantisation for callers that cannot allocate device memory
where they call in (an arena that owns every allocation, a plugin without its host's allocator, a path
that must not synchronise through cudaMalloc). Its column-maximum workspace is a fixed device array
inside the library instead of a caller buffer, so its results must equal those of tbf16_quantize_cols
given a workspace of its own. Bit-exact, like every quantisation test here (integer exponents and
exact fp16 operands).

Two calls in a row: the second has smaller columns than the first, so maxima left in the shared array
by the first call would show up as wrong scales. Collected last (file name) so that a run stopping at
the first failure has run every other test; it also passes alone in a fresh process."""
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_COLS = 65536  # TBF16_NOALLOC_MAX_COLS in include/tbf16_sm100.h


def _call(name, x, t, row_mul, with_ws):
    from tbf16 import _ext as E
    R, K = x.shape
    y = torch.full((R, K), float("nan"), device="cuda", dtype=torch.float16)
    s = torch.full((K,), float("nan"), device="cuda")
    if with_ws:
        ws = torch.empty(K, device="cuda")
        E.call(name, E.ptr(x), R, K, K, t, E.ptr(row_mul), E.ptr(y), K, E.ptr(s), E.ptr(ws), E.stream_ptr())
    else:
        E.call(name, E.ptr(x), R, K, K, t, E.ptr(row_mul), E.ptr(y), K, E.ptr(s), E.stream_ptr())
    torch.cuda.synchronize()
    return y, s


def test_noalloc_matches_allocating_entry_point_twice():
    g = torch.Generator().manual_seed(0)
    first = (torch.randn(512, 1024, generator=g) * 2.0 ** 20).bfloat16().cuda()
    second = (torch.randn(300, 1024, generator=g) * 2.0 ** -6).bfloat16().cuda()  # much smaller columns
    rm = torch.exp2(torch.randint(-4, 5, (300,), generator=g).float()).cuda()
    for x, t, row_mul in ((first, 0, None), (second, -2, rm)):
        y_ref, s_ref = _call("tbf16_quantize_cols", x, t, row_mul, with_ws=True)
        y, s = _call("tbf16_quantize_cols_noalloc", x, t, row_mul, with_ws=False)
        assert torch.equal(s, s_ref)
        assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))


def test_noalloc_rejects_more_columns_than_its_array():
    from tbf16 import _ext as E
    x = torch.zeros(2, MAX_COLS + 8, device="cuda", dtype=torch.bfloat16)
    y = torch.empty_like(x, dtype=torch.float16)
    s = torch.empty(MAX_COLS + 8, device="cuda")
    st = E.lib().tbf16_quantize_cols_noalloc(E.ptr(x), 2, MAX_COLS + 8, MAX_COLS + 8, 0, None, E.ptr(y),
                                             MAX_COLS + 8, E.ptr(s), E.stream_ptr())
    assert st == 1  # TBF16_ERR_INVALID
