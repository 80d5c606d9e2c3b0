"""Failure detection on the GPU without a GPU fault: a bounded wait that runs out returns an error status
the host reads, and the context stays usable afterwards. The wait is the helper every pipelined kernel
(GEMMs, attention) uses, run by tbf16_selftest_bounded_wait on an mbarrier that nothing arrives on, with
a 1 ms limit in place of the kernels' 2 s."""
import pytest
import torch

import inputs
from helpers import rel_err

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports():
    from tbf16 import _ext
    torch.cuda.init()
    assert _ext.device_status(reset=True) == 0
    _ext.call("tbf16_selftest_bounded_wait", 1_000_000, _ext.stream_ptr())
    torch.cuda.synchronize()  # the kernel returned: no hang, no fault
    bits = _ext.device_status(reset=True)
    assert bits & 1, f"timeout bit not set (status bits {bits})"
    assert _ext.device_status(reset=False) == 0  # cleared by the reset


def test_context_usable_after_a_timeout():
    from tbf16 import _ext, ops
    _ext.call("tbf16_selftest_bounded_wait", 50_000, _ext.stream_ptr())
    assert _ext.device_status(reset=True) & 1
    x = inputs.gemm_x(512, 1024, seed=11, device="cuda")
    w = inputs.gemm_w(768, 1024, seed=12, device="cuda")
    y = ops.scaled_linear(x, *ops.prepare_weight(w))
    assert rel_err(y, x.double() @ w.double().t()) < 2e-3
    assert _ext.device_status(reset=True) == 0


def test_selftest_rejects_out_of_range_limits():
    from tbf16 import _ext
    for bad in (0, 2_000_000_000):
        with pytest.raises(RuntimeError):
            _ext.call("tbf16_selftest_bounded_wait", bad, _ext.stream_ptr())
