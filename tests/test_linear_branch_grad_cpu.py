"""The linear branch's differentiable stages (ops/linear_branch_grad.py) on CPU: the adjoint
recurrence of the two scans and the SPD-factor backward against numerical gradients
(float64 gradcheck) and against autograd through the fp32 oracles."""
import pytest
import torch

from vdn_minimax_h3_b200.models import scan as scan_ref
from vdn_minimax_h3_b200.models.delta_rule import DELTA_BACKENDS, VdnDelta, VdnScaledDelta
from vdn_minimax_h3_b200.ops import linear_branch_grad as lbg


def _scan_inputs(F, n, d, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    trans = 0.3 * torch.randn(F, n, d, d, generator=g, dtype=dtype)
    inj = torch.randn(F, n, d, d, generator=g, dtype=dtype)
    start = torch.randn(n, d, d, generator=g, dtype=dtype)
    return trans, inj, start


@pytest.mark.parametrize("with_start", [False, True])
@pytest.mark.parametrize("F", [1, 2, 5])
def test_scans_gradcheck(F, with_start):
    trans, inj, start = _scan_inputs(F, 2, 4, torch.float64)
    args = [trans.requires_grad_(), inj.requires_grad_()]
    if with_start:
        args.append(start.requires_grad_())

    def f(*a):
        p, s = lbg.scans(*a)
        return p, s

    assert torch.autograd.gradcheck(f, tuple(args), eps=1e-6, atol=1e-7, rtol=1e-5)


@pytest.mark.parametrize("with_start", [False, True])
def test_scans_match_oracle_autograd(with_start):
    trans, inj, start = _scan_inputs(7, 3, 16, torch.float32, seed=1)
    st = start if with_start else None
    gp, gs = torch.randn(2, 7, 3, 16, 16, generator=torch.Generator().manual_seed(2))
    leaves = [t.clone().requires_grad_() for t in (trans, inj, start)]
    p, s = lbg.scans(leaves[0], leaves[1], leaves[2] if with_start else None)
    ((p * gp).sum() + (s * gs).sum()).backward()
    ref = [t.clone().requires_grad_() for t in (trans, inj, start)]
    pr, sr = scan_ref.run_scans(ref[0], ref[1], ref[2] if with_start else None)
    ((pr * gp).sum() + (sr * gs).sum()).backward()
    torch.testing.assert_close(p, pr, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(s, sr, rtol=1e-5, atol=1e-5)
    n = 3 if with_start else 2
    for a, b in zip(leaves[:n], ref[:n]):
        torch.testing.assert_close(a.grad, b.grad, rtol=1e-4, atol=1e-4)
    if not with_start:
        assert st is None and leaves[2].grad is None


def _factor_inputs(F, n, d, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(F, n, 3 * d, d, generator=g, dtype=dtype) / d ** 0.5
    A = k.transpose(-1, -2) @ k                 # SPD statistics
    A = 0.5 * (A + A.transpose(-1, -2))
    B = torch.randn(F, n, d, d, generator=g, dtype=dtype)
    alpha = torch.rand(F, n, d, generator=g, dtype=dtype) * 0.5 + 0.4
    return alpha, A, B


@pytest.mark.parametrize("backend", [VdnDelta(), VdnScaledDelta(64)])
def test_vdn_factor_gradcheck(backend):
    alpha, A, B = _factor_inputs(2, 2, 5, torch.float64)
    A0 = A.clone()

    def f(alpha, Araw, B):
        A = 0.5 * (Araw + Araw.transpose(-1, -2))   # the statistics are symmetrised upstream
        return lbg.vdn_factor(backend, alpha, A, B)

    args = (alpha.requires_grad_(), A0.requires_grad_(), B.requires_grad_())
    assert torch.autograd.gradcheck(f, args, eps=1e-6, atol=1e-7, rtol=1e-5)


def test_vdn_factor_matches_oracle_autograd():
    backend = DELTA_BACKENDS["vdn_scaled"](32)
    alpha, A, B = _factor_inputs(3, 2, 16, torch.float32, seed=3)
    g = torch.Generator().manual_seed(4)
    gt, gi = torch.randn(2, 3, 2, 16, 16, generator=g)

    def run(fn):
        leaves = [t.clone().requires_grad_() for t in (alpha, A, B)]
        Asym = 0.5 * (leaves[1] + leaves[1].transpose(-1, -2))
        t, i = fn(leaves[0], Asym, leaves[2])
        ((t * gt).sum() + (i * gi).sum()).backward()
        return (t, i), [x.grad for x in leaves]

    (t, i), grads = run(lambda a, A_, B_: lbg.vdn_factor(backend, a, A_, B_))
    (tr, ir), ref = run(backend.factor_apply)
    torch.testing.assert_close(t, tr, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(i, ir, rtol=1e-4, atol=1e-5)
    for a, b in zip(grads, ref):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-4)
