"""The C-ABI library loads without a GPU and exports every entry point include/*.h declares, and
the ctypes signature table covers each of them (no compute calls here)."""
import ctypes
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(tbf16_[a-z0-9_]+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    from tbf16 import _ext
    lib = _ext.lib()
    names = declared_symbols()
    assert len(names) >= 12
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from tbf16 import _ext
    names = declared_symbols() - {"tbf16_abi_version", "tbf16_status_string"}
    table = set(_ext.SIGNATURES) | set(_ext.SIGNATURES_I64)
    assert names <= table, sorted(names - table)


def test_status_strings_and_version():
    from tbf16 import _ext
    lib = _ext.lib()
    assert lib.tbf16_abi_version() >= 100
    for code in range(8):
        assert lib.tbf16_status_string(code)


def test_no_device_is_an_error_not_a_fallback():
    """Without an sm_100 device every entry point returns a status instead of computing on the CPU."""
    import torch
    from tbf16 import _ext
    if torch.cuda.is_available():
        return
    x = torch.zeros(8, 8, dtype=torch.bfloat16)
    s = torch.zeros(8)
    st = _ext.lib().tbf16_row_scale(_ext.ptr(x), 8, 8, 8, 15, 0, _ext.ptr(s), None, None, 0, None)
    assert st == 5  # TBF16_ERR_DEVICE


def test_ops_raise_without_cuda_tensors():
    import pytest
    import torch
    from tbf16 import ops
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        ops.quantize_rows(x)
