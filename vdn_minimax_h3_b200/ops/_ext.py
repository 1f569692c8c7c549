"""Loader for the package's compiled sm_100a extension (`vdn_minimax_h3_b200._C`).

The extension is built in place (`python setup.py build_ext --inplace`, or
`__graft_entry__.build()`), so the `.so` lives inside the package directory. CUDA tensors
always go through it: if it is missing on a machine that has a GPU, `ext()` raises instead
of quietly running some other implementation. CPU tensors never reach it -- the CPU path
of every op is the fp32 PyTorch oracle the kernels are tested against.
"""
import importlib
import os

import torch

_EXT = None
_ERR = {}
LAUNCHES = [0]   # kernel launches issued through the extension (bench.py reads this)
# Checked launches (VDN_CHECKED=1, or set_checked(True)): every extension call is followed by
# a device synchronise, the CUDA error query and the device error word, and a failure is
# raised naming the call, so an asynchronous fault or an expired bounded wait is pinned to
# the launch that caused it instead of surfacing at some later synchronisation. Slow: a
# debugging mode for small shapes (compute-sanitizer is not available on this hardware pool).
CHECKED = [os.environ.get("VDN_CHECKED", "0") not in ("", "0")]


def set_checked(on=True):
    CHECKED[0] = bool(on)


def _launch_device(args):
    for a in args:
        if getattr(a, "is_cuda", False):
            return a.device
    return None


def _check_args(name, args):
    devs = {str(a.device) for a in args if isinstance(a, torch.Tensor) and a.is_cuda}
    if len(devs) > 1:
        raise ValueError(f"{name}: CUDA tensors on several devices {sorted(devs)}")


def _check_after(name, args):
    device = _launch_device(args)
    if device is None:
        return
    try:
        torch.cuda.synchronize(device)
    except RuntimeError as exc:
        raise KernelError(f"{name}: CUDA error after the launch: {exc}") from exc
    try:
        check_device_error(device)
    except KernelError as exc:
        raise KernelError(f"{name}: {exc}") from exc


class _Counted:
    """The extension module, counting every kernel-launching call made through it."""

    def __init__(self, mod):
        self._mod = mod
        self._cache = {}

    def __getattr__(self, name):
        fn = self._cache.get(name)
        if fn is None:
            raw = getattr(self._mod, name)

            def fn(*args, _raw=raw, _name=name):
                LAUNCHES[0] += 1
                if not CHECKED[0]:
                    return _raw(*args)
                _check_args(_name, args)
                out = _raw(*args)
                _check_after(_name, args)
                return out
            self._cache[name] = fn
        return fn


class KernelError(RuntimeError):
    """A kernel reported a failure through its device error word."""


ERROR_NAMES = {
    1: "TMA producer wait timed out",
    2: "MMA issuer wait timed out",
    3: "epilogue wait timed out",
    4: "peer flag wait timed out",
    5: "bad argument",
    6: "softmax wait timed out",
}


def ext():
    """The compiled module. Raises ImportError with the build command when absent."""
    global _EXT
    if _EXT is None:
        try:
            _EXT = _Counted(importlib.import_module("vdn_minimax_h3_b200._C"))
        except ImportError as exc:  # pragma: no cover - depends on the build
            raise ImportError(
                "vdn_minimax_h3_b200._C is not built; run `python setup.py build_ext --inplace` "
                "(or __graft_entry__.build()). CUDA tensors have no other implementation."
            ) from exc
    return _EXT


def available():
    try:
        ext()
        return True
    except ImportError:
        return False


def error_word(device):
    """The per-device int32 word the kernels write a failure code into."""
    device = torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    word = _ERR.get(key)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _ERR[key] = word
    return word


def check_device_error(device=None, reset=True):
    """Synchronise and raise KernelError if any kernel on `device` recorded a failure."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    word = error_word(device)
    code = int(word.item())
    if code:
        if reset:
            word.zero_()
        raise KernelError(f"device kernel error {code}: {ERROR_NAMES.get(code, 'unknown')}")
