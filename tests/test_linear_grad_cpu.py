"""CPU checks of the training-Linear wiring: the layout GEMM's fp32 oracle for all four
operand layouts, the autograd Function's gradients against F.linear, and the routing."""
import torch
import torch.nn as nn
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops import gemm, linear_grad


def test_matmul_layout_oracle_all_layouts():
    g = torch.Generator().manual_seed(0)
    M, N, K = 24, 40, 16
    a = torch.randn(M, K, generator=g)
    b = torch.randn(N, K, generator=g)
    ref = a @ b.t()
    for a_mn in (False, True):
        for b_mn in (False, True):
            aa = a.t().contiguous() if a_mn else a
            bb = b.t().contiguous() if b_mn else b
            y = gemm.matmul_layout(aa, bb, a_mn=a_mn, b_mn=b_mn)
            assert y.shape == (M, N)
            torch.testing.assert_close(y, ref, rtol=1e-5, atol=1e-5)
            acc = torch.ones(M, N)
            gemm.matmul_layout(aa, bb, a_mn=a_mn, b_mn=b_mn, out=acc, accumulate=True)
            torch.testing.assert_close(acc, ref + 1, rtol=1e-5, atol=1e-5)


def test_dgrad_wgrad_formulas():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(30, 16, generator=g)
    w = torch.randn(8, 16, generator=g)
    dy = torch.randn(30, 8, generator=g)
    torch.testing.assert_close(gemm.linear_dgrad(dy, w), dy @ w)
    torch.testing.assert_close(gemm.linear_wgrad(dy, x), dy.t() @ x)


def test_kernel_linear_function_grads_match_autograd():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 7, 16, generator=g, requires_grad=True)
    w = torch.randn(24, 16, generator=g, requires_grad=True)
    b = torch.randn(24, generator=g, requires_grad=True)
    up = torch.randn(2, 7, 24, generator=g)
    y = linear_grad._KernelLinear.apply(x.reshape(-1, 16), w, b).view(2, 7, 24)
    y.backward(up)
    got = [t.grad.clone() for t in (x, w, b)]
    for t in (x, w, b):
        t.grad = None
    F.linear(x, w, b).backward(up)
    for a, r in zip(got, (x.grad, w.grad, b.grad)):
        torch.testing.assert_close(a, r, rtol=1e-5, atol=1e-5)


def test_route_training_linears_falls_back_on_cpu():
    torch.manual_seed(3)
    model = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 8, bias=False))
    ref = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 8, bias=False))
    ref.load_state_dict(model.state_dict())
    assert linear_grad.route_training_linears(model) == 2
    assert linear_grad.route_training_linears(model) == 0        # idempotent
    assert list(model.state_dict()) == list(ref.state_dict())    # names untouched
    x = torch.randn(5, 16)
    before = linear_grad.STATS["fallback"]
    torch.testing.assert_close(model(x), ref(x))
    assert linear_grad.STATS["fallback"] == before + 2           # CPU tensors: F.linear
