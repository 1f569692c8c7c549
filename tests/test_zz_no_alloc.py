"""The allocation-free C entry point vdn_delta_stats_factor_noalloc (csrc/vdn_noalloc.h),
called through its exported C symbol, equals the allocating ops path
(ops.linear_branch.frame_statistics + factor_apply) on two consecutive calls, and rejects
requests above its scratch limit. Collected last, so it also runs after every other test."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from vdn_minimax_h3_b200 import _C
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.vdn_delta_stats_factor_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.vdn_noalloc_read_device_error.restype = ctypes.c_int
    lib.vdn_noalloc_read_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
    lib.vdn_noalloc_error_string.restype = ctypes.c_char_p
    lib.vdn_noalloc_error_string.argtypes = [ctypes.c_int]
    return lib


def _inputs(F, S, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.nn.functional.normalize(torch.randn(F * S, H, 128, device="cuda", generator=g), dim=-1)
    v = torch.randn(F * S, H, 128, device="cuda", generator=g)
    beta = torch.sigmoid(torch.randn(F * S, H, device="cuda", generator=g))
    alpha = torch.rand(F, H, 128, device="cuda", generator=g) * 0.5 + 0.5
    return (k.to(torch.bfloat16).reshape(F * S, H * 128), v.to(torch.bfloat16).reshape(F * S, H * 128),
            beta, alpha)


def test_noalloc_matches_allocating_path_twice():
    from vdn_minimax_h3_b200.models.delta_rule import VdnDelta
    from vdn_minimax_h3_b200.ops import linear_branch as lb
    from vdn_minimax_h3_b200.ops._ext import check_device_error
    lib = _lib()
    F, S, H = 6, 200, 4
    backend = VdnDelta(S)
    for call in range(2):
        k, v, beta, alpha = _inputs(F, S, H, seed=call)
        A, B = lb.frame_statistics(k.view(F, S, H, 128), v.view(F, S, H, 128), beta.view(F, S, H))
        ref_t, ref_i = lb.factor_apply(backend, alpha, A, B)
        trans = torch.empty(F, H, 128, 128, device="cuda")
        inj = torch.empty_like(trans)
        stream = torch.cuda.current_stream().cuda_stream
        rc = lib.vdn_delta_stats_factor_noalloc(
            k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), beta.contiguous().data_ptr(),
            alpha.contiguous().data_ptr(), F, S, H, float(backend.a_scale), float(backend.b_scale),
            trans.data_ptr(), inj.data_ptr(), stream)
        assert rc == 0, lib.vdn_noalloc_error_string(rc)
        torch.cuda.synchronize()
        code = ctypes.c_int(-1)
        assert lib.vdn_noalloc_read_device_error(ctypes.byref(code)) == 0 and code.value == 0
        check_device_error()
        assert torch.equal(trans, ref_t) and torch.equal(inj, ref_i)


def test_noalloc_rejects_oversize():
    lib = _lib()
    F, S, H = 33, 8, 4          # 132 matrices > the 128 of the scratch
    k, v, beta, alpha = _inputs(F, S, H, seed=3)
    out = torch.empty(F, H, 128, 128, device="cuda")
    rc = lib.vdn_delta_stats_factor_noalloc(
        k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0), beta.data_ptr(), alpha.data_ptr(),
        F, S, H, 1.0, 1.0, out.data_ptr(), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"VDN_NOALLOC_MAX_MATS" in lib.vdn_noalloc_error_string(rc)
