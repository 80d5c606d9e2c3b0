"""The attention backward's overflow retry (reference tbf16/autograd.py:177-189), on the host with the
kernel call replaced by a stub: the stub raises the kernel's non-finite flag for the first k attempts.
Each retry must lower the dO target exponent t_do by 8; the call succeeds while k < 6 and raises
FloatingPointError when all six attempts overflow. No GPU: the tensors are CPU tensors and nothing
is launched."""
import ctypes
import math

import pytest
import torch

# position of t_do and of the flag pointer in tbf16_attn_bwd's argument list (include/tbf16_sm100.h)
T_DO_ARG, FLAG_ARG = 25, 30


class _StubKernel:
    def __init__(self, overflowing_attempts):
        self.left = overflowing_attempts
        self.t_do = []

    def __call__(self, name, *args):
        assert name == "tbf16_attn_bwd"
        self.t_do.append(args[T_DO_ARG])
        if self.left > 0:
            self.left -= 1
            ctypes.c_int.from_address(args[FLAG_ARG].value).value = 1  # the kernel's non-finite flag


class _StubLib:
    @staticmethod
    def tbf16_attn_bwd_workspace_size(*_):
        return 64


def _run(monkeypatch, k, check=True):
    from tbf16 import autograd as ag
    stub = _StubKernel(k)
    monkeypatch.setattr(ag, "call", stub)
    monkeypatch.setattr(ag, "lib", lambda: _StubLib())
    monkeypatch.setattr(ag, "stream_ptr", lambda dev=None: ctypes.c_void_p(0))
    monkeypatch.setattr(ag, "CHECK_OVERFLOW", check)
    B, H, S, D = 1, 2, 16, 64
    q16, k16, v16, o16 = (torch.zeros(B, H, S, D, dtype=torch.float16) for _ in range(4))
    lse = torch.zeros(B, H, 128)
    a, ev = torch.zeros((), dtype=torch.int32), torch.zeros(B, H, dtype=torch.int32)
    dout = torch.zeros(B, H, S, D, dtype=torch.bfloat16)
    ag.attn_backward(q16, k16, v16, o16, lse, a, ev, dout, None, False, 0.125, D)
    return stub


@pytest.mark.parametrize("k", [0, 1, 3, 5])
def test_retry_lowers_t_do_by_8_until_finite(monkeypatch, k):
    stub = _run(monkeypatch, k)
    t0 = 12 - math.ceil(math.log2(64))
    assert stub.t_do == [t0 - 8 * i for i in range(k + 1)]


def test_six_overflowing_attempts_raise_floating_point_error(monkeypatch):
    with pytest.raises(FloatingPointError):
        _run(monkeypatch, 6)


def test_check_overflow_off_runs_once(monkeypatch):
    """TBF16_ATTN_CHECK=0 (CHECK_OVERFLOW False): one attempt, no host sync, no retry (as the reference)."""
    stub = _run(monkeypatch, 6, check=False)
    assert len(stub.t_do) == 1
