"""The AdaLN-modulated RMSNorm's training path on a B200: forward kernel + backward kernel
(csrc/norm_bwd.cu) against fp32 autograd through the eager expression, for x and for the
norm weight and the modulation tables (those in PyTorch, when required)."""
import pytest
import torch

from vdn_minimax_h3_b200.ops import norm_grad
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


class _Norm(torch.nn.Module):
    def __init__(self, w, eps):
        super().__init__()
        self.weight = torch.nn.Parameter(w)
        self.eps = eps

    def forward(self, x):
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), self.weight.to(x.dtype), self.eps)


@pytest.mark.parametrize("T,D,n,grads_all", [(300, 512, 3, True), (64, 5376, 2, False)])
def test_adaln_norm_backward_kernel(T, D, n, grads_all):
    g = torch.Generator().manual_seed(T + D)
    x = torch.randn(1, T, D, generator=g).to(torch.bfloat16).cuda()
    w = (1 + 0.1 * torch.randn(D, generator=g)).cuda()
    shift = (0.3 * torch.randn(n, D, generator=g)).to(torch.bfloat16).cuda()
    scale = (0.3 * torch.randn(n, D, generator=g)).to(torch.bfloat16).cuda()
    idx = torch.randint(0, n, (T,), generator=g).cuda()
    up = torch.randn(1, T, D, generator=g).to(torch.bfloat16).cuda()
    norm = _Norm(w.clone(), 1e-6).cuda()
    norm.weight.requires_grad_(grads_all)
    xk = x.clone().requires_grad_()
    sk, ck = shift.clone().requires_grad_(grads_all), scale.clone().requires_grad_(grads_all)
    out = norm_grad.adaln_modulated_norm(norm, xk, sk, ck, idx)
    (out.float() * up.float()).sum().backward()
    check_device_error()
    assert out.dtype == torch.bfloat16 and out.shape == x.shape
    ref_norm = _Norm(w.clone(), 1e-6).cuda()
    xr = x.float().requires_grad_()
    sr, cr = shift.float().requires_grad_(), scale.float().requires_grad_()
    ref = ref_norm(xr) * (1.0 + cr.index_select(0, idx)) + sr.index_select(0, idx)
    (ref * up.float()).sum().backward()
    assert _rel(out, ref) < 1e-2
    assert _rel(xk.grad, xr.grad) < 1e-2
    if grads_all:
        assert _rel(norm.weight.grad, ref_norm.weight.grad) < 1e-2
        assert _rel(sk.grad, sr.grad) < 1e-2
        assert _rel(ck.grad, cr.grad) < 1e-2


def test_adaln_norm_same_path_with_and_without_grad():
    """A no-grad forward (the teacher) and a graph-recording forward (the student) run the
    same kernel, bit for bit. The kernel rounds once where the eager bf16 expression rounds
    after every op, so it is checked to be at least as close to the fp32 result as eager is,
    and close to eager itself."""
    g = torch.Generator().manual_seed(7)
    T, D, n = 257, 1024, 3
    x = torch.randn(1, T, D, generator=g).to(torch.bfloat16).cuda()
    norm = _Norm((1 + 0.1 * torch.randn(D, generator=g)).cuda(), 1e-6).cuda()
    shift = (0.3 * torch.randn(n, D, generator=g)).to(torch.bfloat16).cuda()
    scale = (0.3 * torch.randn(n, D, generator=g)).to(torch.bfloat16).cuda()
    idx = torch.randint(0, n, (T,), generator=g).cuda()
    with torch.no_grad():
        teacher = norm_grad.adaln_modulated_norm(norm, x, shift, scale, idx)
    student = norm_grad.adaln_modulated_norm(norm, x.clone().requires_grad_(), shift, scale, idx)
    check_device_error()
    assert torch.equal(teacher, student.detach())
    with torch.no_grad():
        eager = norm(x) * (1.0 + scale.index_select(0, idx)) + shift.index_select(0, idx)
        xf = x.float()
        exact = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * norm.weight
                 * (1.0 + scale.float().index_select(0, idx)) + shift.float().index_select(0, idx))
    assert _rel(teacher, exact) <= _rel(eager, exact) * 1.05
    assert _rel(teacher, eager) < 8e-3
