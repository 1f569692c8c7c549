"""tcgen05 GEMM kernels vs an fp32 PyTorch reference of the same op."""
import pytest
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops import gemm
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu

SHAPES = [(128, 256, 64), (256, 512, 128), (300, 200, 136), (1000, 768, 1024),
          (129, 264, 72), (4096, 5376, 512)]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_store(M, N, K):
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(N, device="cuda")
    y = gemm.linear(x, w, b)
    check_device_error()
    ref = F.linear(x.float(), w.float(), b)
    assert _rel(y, ref) < 8e-3


@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (333, 304, 200)])
def test_gemm_accumulate(M, N, K):
    torch.manual_seed(1)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    out = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    ref = out.float() + x.float() @ w.float().t()
    gemm.linear(x, w, out=out, accumulate=True)
    check_device_error()
    assert _rel(out, ref) < 8e-3


@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (333, 768, 200)])
def test_gemm_residual(M, N, K):
    torch.manual_seed(2)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(N, device="cuda")
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    table = torch.randn(6, N, device="cuda", dtype=torch.bfloat16)
    idx = torch.randint(0, 6, (M,), device="cuda", dtype=torch.int32)
    ref = res.float() + table.float()[idx.long()] * F.linear(x.float(), w.float(), b)
    gemm.linear_gated_residual(x, w, b, res, table, idx)
    check_device_error()
    assert _rel(res, ref) < 8e-3


@pytest.mark.parametrize("M,I,K", [(256, 256, 128), (300, 512, 200)])
def test_gemm_swiglu(M, I, K):
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * I, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(2 * I, device="cuda")
    wi, bi = gemm.interleave_swiglu_rows(w, b)
    y = gemm.linear_swiglu(x, wi, bi)
    check_device_error()
    h = F.linear(x.float(), w.float(), b)
    ref = h[:, :I] * F.silu(h[:, I:])
    assert _rel(y, ref) < 8e-3
