"""Checked launches (ops/_ext.py, VDN_CHECKED=1): each extension call is followed by a
synchronise and the error-word check, and a failure names the call. Exercised on CPU with a
stand-in extension module and a stand-in CUDA argument."""
import pytest

from vdn_minimax_h3_b200.ops import _ext


class _FakeMod:
    def __init__(self):
        self.calls = []

    def lb_scan(self, *args):
        self.calls.append(args)
        return "ran"


class _CudaLike:
    is_cuda = True
    device = "cuda:0"


@pytest.fixture
def checked():
    old = _ext.CHECKED[0]
    _ext.set_checked(True)
    yield
    _ext.set_checked(old)


def test_unchecked_calls_pass_through():
    mod = _FakeMod()
    wrapped = _ext._Counted(mod)
    n0 = _ext.LAUNCHES[0]
    old = _ext.CHECKED[0]
    _ext.set_checked(False)
    try:
        assert wrapped.lb_scan(_CudaLike()) == "ran"
    finally:
        _ext.set_checked(old)
    assert _ext.LAUNCHES[0] == n0 + 1 and len(mod.calls) == 1


def test_checked_call_names_the_failing_launch(checked, monkeypatch):
    synced = []
    monkeypatch.setattr(_ext.torch.cuda, "synchronize", lambda d=None: synced.append(d))

    def failing(device=None, reset=True):
        raise _ext.KernelError("device kernel error 1: TMA producer wait timed out")

    monkeypatch.setattr(_ext, "check_device_error", failing)
    wrapped = _ext._Counted(_FakeMod())
    with pytest.raises(_ext.KernelError, match=r"^lb_scan: device kernel error 1"):
        wrapped.lb_scan(_CudaLike())
    assert synced == ["cuda:0"]


def test_checked_call_reports_async_cuda_errors(checked, monkeypatch):
    def boom(d=None):
        raise RuntimeError("CUDA error: an illegal memory access was encountered")

    monkeypatch.setattr(_ext.torch.cuda, "synchronize", boom)
    wrapped = _ext._Counted(_FakeMod())
    with pytest.raises(_ext.KernelError, match=r"^lb_scan: CUDA error after the launch"):
        wrapped.lb_scan(_CudaLike())


def test_checked_call_without_cuda_arguments_skips_the_device(checked, monkeypatch):
    monkeypatch.setattr(_ext.torch.cuda, "synchronize",
                        lambda d=None: pytest.fail("no CUDA argument: nothing to synchronise"))
    wrapped = _ext._Counted(_FakeMod())
    assert wrapped.lb_scan(3, "x") == "ran"
