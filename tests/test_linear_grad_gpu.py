"""Training Linears on a B200: the bf16 tcgen05 GEMM with MN-major operands (the input and
weight gradients of a Linear, read in their stored layouts) against fp32 matmuls, and the
routed nn.Linear's forward / dgrad / wgrad / bias gradient against fp32 autograd, with a
budget set by eager bf16 F.linear (cuBLAS) on the same inputs."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops import gemm, linear_grad
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


# M, N, K with tails on every axis (M vs 128, N vs 256 and vs the 64-wide MN boxes, K vs 64),
# a long contraction (the wgrad shape: K = tokens), and an N below one box.
SHAPES = [(200, 328, 136), (256, 512, 4136), (136, 40, 72)]


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_matmul_layout_vs_fp32(a_mn, b_mn, shape):
    M, N, K = shape
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, generator=g).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    aa = (a.t().contiguous() if a_mn else a).cuda()
    bb = (b.t().contiguous() if b_mn else b).cuda()
    y = gemm.matmul_layout(aa, bb, a_mn=a_mn, b_mn=b_mn)
    base = torch.randn(M, N, generator=g).to(torch.bfloat16)
    acc = base.cuda()
    gemm.matmul_layout(aa, bb, a_mn=a_mn, b_mn=b_mn, out=acc, accumulate=True)
    torch.cuda.synchronize()
    check_device_error()
    # one bf16 rounding of an fp32 accumulator: <= 2^-9 relative per element
    assert _rel(y, ref) < 4e-3
    assert _rel(acc, ref + base.float()) < 4e-3


def test_matmul_layout_strided_views():
    # operands that are row-strided views (a column slice of a wider buffer)
    g = torch.Generator().manual_seed(7)
    wide = torch.randn(520, 384, generator=g).to(torch.bfloat16).cuda()
    dy = wide[:, :200]             # [T=520, out=200], row stride 384
    x = wide[:, 200:384]           # [T=520, in=184], row stride 384, offset 400 B
    dw = gemm.linear_wgrad(dy, x)
    torch.cuda.synchronize()
    check_device_error()
    assert _rel(dw, dy.float().t() @ x.float()) < 4e-3


@pytest.mark.parametrize("bias", [True, False])
def test_kernel_linear_grads_vs_fp32_autograd(bias):
    g = torch.Generator().manual_seed(11)
    T, din, dout = 2100, 392, 200
    x0 = (torch.randn(3, T // 3, din, generator=g)).to(torch.bfloat16)
    w0 = (torch.randn(dout, din, generator=g) * din ** -0.5).to(torch.bfloat16)
    b0 = torch.randn(dout, generator=g).to(torch.bfloat16) if bias else None
    up = torch.randn(3, T // 3, dout, generator=g).to(torch.bfloat16)

    def run(fn, dev, dtype):
        ts = [t.to(dev, dtype).requires_grad_() for t in (x0, w0) + ((b0,) if bias else ())]
        y = fn(ts[0], ts[1], ts[2] if bias else None)
        y.backward(up.to(dev, dtype))
        return [y.detach()] + [t.grad for t in ts]

    before = linear_grad.STATS["kernel"]
    ours = run(linear_grad.kernel_linear, "cuda", torch.bfloat16)
    torch.cuda.synchronize()
    check_device_error()
    assert linear_grad.STATS["kernel"] == before + 1
    eager = run(F.linear, "cuda", torch.bfloat16)
    ref = run(F.linear, "cpu", torch.float32)
    for name, o, e, r in zip(["y", "dx", "dw", "db"], ours, eager, ref):
        eo, ee = _rel(o, r), _rel(e, r)
        assert eo <= 1.5 * ee + 1e-3, (name, eo, ee)


def test_routed_module_matches_eager_grads():
    torch.manual_seed(5)
    model = nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 256)).cuda().to(torch.bfloat16)
    ref = nn.Sequential(nn.Linear(256, 512), nn.GELU(), nn.Linear(512, 256)).cuda().to(torch.bfloat16)
    ref.load_state_dict(model.state_dict())
    assert linear_grad.route_training_linears(model) == 2
    x = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16)
    model(x).float().square().mean().backward()
    ref(x).float().square().mean().backward()
    torch.cuda.synchronize()
    check_device_error()
    for (n, p), (_, q) in zip(model.named_parameters(), ref.named_parameters()):
        assert _rel(p.grad, q.grad) < 2e-2, n
