"""The differentiable AdaLN norm (ops/norm_grad.py) on CPU: the dispatcher falls back to the
eager expression off the GPU, and the autograd Function's own logic (modulation table,
row indices, the optional weight / shift / scale gradients) matches autograd of the eager
expression when the extension's dx is computed by the same formula in PyTorch."""
import torch

from vdn_minimax_h3_b200.ops import _ext, norm_grad


class _Norm(torch.nn.Module):
    def __init__(self, w, eps=1e-6):
        super().__init__()
        self.weight = torch.nn.Parameter(w)
        self.eps = eps

    def forward(self, x):
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), self.weight.to(x.dtype), self.eps)


class _StubExt:
    """dx = r g - (r^3 / D) x sum(g x), g = dy w (1 + scale[idx]) -- what norm_bwd.cu computes."""

    def adaln_rmsnorm_bwd(self, x, dy, w, eps, table, scale_col, idx, dx):
        xf, g = x.float(), dy.float()
        D = x.shape[1]
        if w is not None:
            g = g * w
        g = g * (1.0 + table[:, scale_col:scale_col + D].float()[idx.long()])
        r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        dx.copy_(r * g - r.pow(3) / D * xf * (g * xf).sum(-1, keepdim=True))


def _data(T=40, D=64, n=3):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, T, D, generator=g).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(D, generator=g)
    shift = (0.3 * torch.randn(n, D, generator=g)).to(torch.bfloat16)
    scale = (0.3 * torch.randn(n, D, generator=g)).to(torch.bfloat16)
    idx = torch.randint(0, n, (T,), generator=g)
    up = torch.randn(1, T, D, generator=g)
    return x, w, shift, scale, idx, up


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_cpu_rows_take_the_eager_expression():
    x, w, shift, scale, idx, _ = _data()
    norm = _Norm(w)
    out = norm_grad.adaln_modulated_norm(norm, x, shift, scale, idx)
    ref = norm(x) * (1.0 + scale.index_select(0, idx)) + shift.index_select(0, idx)
    assert torch.equal(out, ref)


def test_function_gradients_match_eager_autograd(monkeypatch):
    monkeypatch.setattr(_ext, "ext", lambda: _StubExt())
    x, w, shift, scale, idx, up = _data()
    norm = _Norm(w.clone())
    leaves = [x.clone().requires_grad_(), shift.clone().requires_grad_(),
              scale.clone().requires_grad_()]
    out = norm_grad._AdaLNNorm.apply(leaves[0].view(-1, x.shape[-1]), norm.weight, leaves[1],
                                     leaves[2], idx, norm.eps)
    (out.float() * up.view(out.shape)).sum().backward()
    ref_norm = _Norm(w.clone())
    rl = [x.float().requires_grad_(), shift.float().requires_grad_(),
          scale.float().requires_grad_()]
    ref = ref_norm(rl[0]) * (1.0 + rl[2].index_select(0, idx)) + rl[1].index_select(0, idx)
    (ref * up).sum().backward()
    assert _rel(out.view(ref.shape), ref) < 1e-2
    for a, b in zip(leaves, rl):
        assert _rel(a.grad, b.grad) < 1e-2
    assert _rel(norm.weight.grad, ref_norm.weight.grad) < 1e-2
