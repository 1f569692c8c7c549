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


def _rope_tables(M, device):
    pos = torch.stack([torch.arange(M) // 97, (torch.arange(M) // 7) % 13, torch.arange(M) % 7], 1)
    from vdn_minimax_h3_b200.models.h3 import RotaryEmbedding3D
    cos, sin = RotaryEmbedding3D((32, 48, 48))(pos.to(device))
    return cos.contiguous(), sin.contiguous()


@pytest.mark.parametrize("M", [1000, 4096])
def test_gemm_routed_qkv(M):
    """Routed epilogue: raw columns to a packed buffer, QK-norm + RoPE'd heads to q/k
    buffers, a replicated field to a third plane; vs fp32 projection + qk_prep oracle."""
    from vdn_minimax_h3_b200.ops.norm import qk_prep_reference
    torch.manual_seed(5)
    K = 512
    cols = {"q": (0, 256), "k": (256, 512), "v": (512, 768), "sgate": (768, 776),
            "beta": (776, 784), "ghid": (784, 848)}
    N = 848
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / K ** 0.5
    b = torch.randn(N, device="cuda") * 0.1
    nq = torch.rand(128, device="cuda") + 0.5
    nk = torch.rand(128, device="cuda") + 0.5
    cos, sin = _rope_tables(M, "cuda")
    raw = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    q = torch.zeros(M, 256, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(M, 256, device="cuda", dtype=torch.bfloat16)
    gh = torch.zeros(M, 64, device="cuda", dtype=torch.bfloat16)
    route = gemm.ColumnRoute(N, planes=3)
    route.place(0, raw).place(0, q, plane=1).place(256, k, plane=1).place(784, gh, plane=2)
    gemm.linear_routed(x, w, b, route, cols["q"], cols["k"], nq, nk, 1e-6, cos, sin)
    torch.cuda.synchronize()
    check_device_error()
    ref = F.linear(x.float(), w.float(), b)
    assert _rel(raw, ref) < 8e-3
    assert torch.equal(gh, raw[:, 784:848])
    q_ref = qk_prep_reference(raw[:, 0:256], 2, nq, 1e-6, cos, sin)
    k_ref = qk_prep_reference(raw[:, 256:512], 2, nk, 1e-6, cos, sin)
    assert _rel(q, q_ref) < 8e-3 and _rel(k, k_ref) < 8e-3
    # second call through the cached tables gives the same bits
    q2 = q.clone()
    gemm.linear_routed(x, w, b, route, cols["q"], cols["k"], nq, nk, 1e-6, cos, sin)
    torch.cuda.synchronize()
    assert torch.equal(q, q2)
