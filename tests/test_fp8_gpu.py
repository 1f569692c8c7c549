"""Block-scaled fp8 kernels vs their fp32 oracles (dequantise, matmul in fp32)."""
import pytest
import torch

from vdn_minimax_h3_b200.ops import fp8
from vdn_minimax_h3_b200.ops._ext import check_device_error
from vdn_minimax_h3_b200.ops.gemm import interleave_swiglu_rows

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,K", [(130, 256), (1000, 5376)])
def test_quant_rows_matches_oracle(M, K):
    torch.manual_seed(0)
    x = (torch.randn(M, K, device="cuda") * torch.rand(M, 1, device="cuda") * 10).to(torch.bfloat16)
    q, sf = fp8.quantize_act(x)
    torch.cuda.synchronize()
    qr, sfr = fp8.quantize_act(x.cpu())
    assert torch.equal(fp8.sf_unblock(sf.cpu(), M, K, 128), fp8.sf_unblock(sfr, M, K, 128))
    mism = (q.cpu() != qr).float().mean().item()
    assert mism < 1e-4, mism


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (300, 544, 384), (2048, 5376, 5376)])
def test_gemm_fp8_store(M, N, K):
    torch.manual_seed(1)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(N, device="cuda")
    xq, xsf = fp8.quantize_act(x)
    fw = fp8.Fp8Weight(w, b)
    y = fp8.linear_fp8(xq, xsf, fw)
    torch.cuda.synchronize()
    check_device_error()
    ref = fp8.dequantize(xq, xsf, 128) @ fw.dequantized().t() + b
    assert _rel(y, ref) < 8e-3
    assert _rel(y, x.float() @ w.float().t() + b) < 0.06


def test_gemm_fp8_residual():
    torch.manual_seed(2)
    M, N, K = 333, 512, 256
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / 16
    fw = fp8.Fp8Weight(w)
    xq, xsf = fp8.quantize_act(x)
    res = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    table = torch.randn(3, N, device="cuda", dtype=torch.bfloat16)
    idx = torch.randint(0, 3, (M,), device="cuda", dtype=torch.int32)
    ref = res.float() + table.float()[idx.long()] * (fp8.dequantize(xq, xsf, 128) @ fw.dequantized().t())
    fp8.linear_fp8_gated_residual(xq, xsf, fw, res, table, idx)
    torch.cuda.synchronize()
    check_device_error()
    assert _rel(res, ref) < 8e-3


def test_gemm_fp8_swiglu_quant():
    torch.manual_seed(3)
    M, I, K = 500, 512, 384
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * I, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    wi, _ = interleave_swiglu_rows(w, None, tile=128)
    fw = fp8.Fp8Weight(wi)
    xq, xsf = fp8.quantize_act(x)
    q, sf = fp8.linear_fp8_swiglu(xq, xsf, fw)
    torch.cuda.synchronize()
    check_device_error()
    h = fp8.dequantize(q, sf, 128)
    y = (fp8.dequantize(xq, xsf, 128) @ fw.dequantized().t()).view(M, 2 * I // 128, 2, 64)
    ref = (y[:, :, 0] * torch.nn.functional.silu(y[:, :, 1])).reshape(M, I)
    assert _rel(h, ref) < 0.05
