"""Host-side logic of the public API without a GPU: exports mirror the reference, exponent target
rule, row cache, conversion routing, and that nothing silently computes on the CPU."""
import pytest
import torch
import torch.nn as nn


def test_exports_match_reference_api():
    import tbf16
    ref_all = ["quantize_rows", "scaled_linear", "prepare_weight", "sdpa", "patch", "TuringBF16Mode", "convert",
               "Linear", "TrainLinear", "autograd", "install_sdpa", "uninstall_sdpa", "is_supported_gpu"]
    assert set(ref_all) <= set(tbf16.__all__)
    from tbf16 import attention, autograd, ops
    for mod, names in ((ops, ["quantize_rows", "quantize_rows_shared", "prepare_weight", "scaled_linear", "linear_q",
                               "small_m_linear", "_target_exp", "L1_TARGET", "SMALL_M", "_RowCache"]),
                       (attention, ["head_exp", "head_scale", "prepare_qkv", "expand_heads", "sdpa"]),
                       (autograd, ["quantize_cols", "ScaledLinearFn", "FP32LinearFn", "linear", "ScaledSDPAFn", "sdpa",
                                   "CHECK_OVERFLOW"])):
        for n in names:
            assert hasattr(mod, n), f"{mod.__name__}.{n}"


def test_target_exp_matches_oracle():
    from oracle import oracle as orc
    from tbf16 import ops
    for K in (1, 8, 1000, 4096, 32768, 32769, 65536, 1 << 20):
        assert ops._target_exp(K) == orc.target_exp(K)


def test_row_cache_identity_and_version():
    from tbf16.ops import _RowCache
    cache = _RowCache(size=2)
    calls = []
    x = torch.zeros(3)
    make = lambda: calls.append(1) or len(calls)
    assert cache.get(x, 15, make) == 1
    assert cache.get(x, 15, make) == 1          # hit
    assert cache.get(x, 0, make) == 2           # different target
    x.add_(1)                                   # in-place change bumps the version
    assert cache.get(x, 15, make) == 3


def test_convert_is_noop_without_sm100():
    import tbf16
    if torch.cuda.is_available():
        pytest.skip("needs a machine without an sm_100 GPU")
    m = nn.Sequential(nn.Linear(16, 16).bfloat16())
    with pytest.warns(UserWarning):
        out = tbf16.convert(m)
    assert out is m and type(m[0]) is nn.Linear


def test_convert_train_swaps_class_in_place():
    import tbf16
    m = nn.Sequential(nn.Linear(16, 16), nn.ReLU(), nn.Linear(16, 4))
    params = [id(p) for p in m.parameters()]
    tbf16.convert(m, train=True, sdpa=False, force=True)
    assert type(m[0]) is tbf16.TrainLinear and type(m[2]) is tbf16.TrainLinear
    assert [id(p) for p in m.parameters()] == params
    y = m(torch.randn(2, 16))  # fp32 CPU input: TrainLinear stays native F.linear
    assert y.shape == (2, 4)


def _convert_module():
    import importlib
    return importlib.import_module("tbf16.convert")  # tbf16.convert is also the function's name


def test_sdpa_routing_keeps_cpu_native():
    convert = _convert_module()
    q = k = v = torch.randn(1, 2, 32, 16).bfloat16()
    out = convert._sdpa(q, k, v)
    ref = convert._native_sdpa(q, k, v)
    assert torch.equal(out, ref)


def test_install_uninstall_sdpa():
    import torch.nn.functional as F
    convert = _convert_module()
    native = F.scaled_dot_product_attention
    convert.install_sdpa()
    try:
        assert F.scaled_dot_product_attention is convert._sdpa
    finally:
        convert.uninstall_sdpa()
    assert F.scaled_dot_product_attention is native


def test_patch_mode_counts_native_calls_on_cpu():
    import torch.nn.functional as F
    import tbf16
    with torch.no_grad(), tbf16.patch() as mode:
        F.linear(torch.randn(4, 8).bfloat16(), torch.randn(3, 8).bfloat16())
        q = torch.randn(1, 2, 32, 16).bfloat16()
        F.scaled_dot_product_attention(q, q, q)
    assert mode.stats["sdpa_native"] == 1 and mode.stats["linear"] == 0


def test_no_cpu_compute_path():
    from tbf16 import attention, autograd, ops
    x = torch.randn(8, 16).bfloat16()
    for fn in (lambda: ops.quantize_rows(x), lambda: autograd.quantize_cols(x),
               lambda: attention.head_exp(x.view(1, 1, 8, 16))):
        with pytest.raises(RuntimeError):
            fn()


def test_linear_host_chunks_cover_rows_once():
    """linear_host's chunking: contiguous, covering every row once, no chunk above chunk_rows, short first
    and last chunks when there are several."""
    from tbf16 import ops
    for M, rows in [(8192, 1024), (2053, 1024), (1024, 1024), (1300, 1024), (5, 1024), (1030, 1024), (9000, 512)]:
        ch = ops._host_chunks(M, rows)
        assert ch[0][0] == 0 and sum(n for _, n in ch) == M
        assert all(ch[i][0] + ch[i][1] == ch[i + 1][0] for i in range(len(ch) - 1))
        assert all(0 < n <= rows for _, n in ch)
        if M > rows:
            assert ch[0][1] == rows // 4
