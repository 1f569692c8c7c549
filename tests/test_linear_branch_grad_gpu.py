"""The linear branch's training stages on the GPU: the SPD-factor and scan kernels forward and
the adjoint scan (one prefix-only launch of the scan kernel over 2H stacked recurrences)
backward, against autograd through the fp32 PyTorch recurrences on the same device."""
import pytest
import torch

from vdn_minimax_h3_b200.models import scan as scan_ref
from vdn_minimax_h3_b200.models.delta_rule import VdnDelta, VdnScaledDelta
from vdn_minimax_h3_b200.ops import linear_branch_grad as lbg
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _grads(fn, inputs, upstream):
    leaves = [None if t is None else t.clone().requires_grad_() for t in inputs]
    outs = fn(*leaves)
    sum(((o * g).sum() for o, g in zip(outs, upstream))).backward()
    return outs, [None if t is None else t.grad for t in leaves]


@pytest.mark.parametrize("with_start", [False, True])
@pytest.mark.parametrize("F,H", [(9, 3), (1, 2), (12, 56)])
def test_scan_adjoint_kernel(F, H, with_start):
    g = torch.Generator().manual_seed(F * 100 + H)
    trans = (torch.randn(F, H, 128, 128, generator=g) * 0.06).cuda()
    inj = torch.randn(F, H, 128, 128, generator=g).cuda()
    start = torch.randn(H, 128, 128, generator=g).cuda() if with_start else None
    up = [torch.randn(F, H, 128, 128, generator=g).cuda() for _ in range(2)]
    outs, grads = _grads(lbg.scans, (trans, inj, start), up)
    check_device_error()
    ref_outs, ref_grads = _grads(scan_ref.run_scans, (trans, inj, start), up)
    for a, b in zip(outs, ref_outs):
        assert _rel(a, b) < 1e-4
    for a, b in zip(grads, ref_grads):
        if b is None:
            assert a is None
        else:
            assert _rel(a, b) < 1e-4


@pytest.mark.parametrize("backend", [VdnDelta(), VdnScaledDelta(256)])
def test_vdn_factor_kernel_grad(backend):
    g = torch.Generator().manual_seed(7)
    F, H, S = 4, 3, 256
    k = torch.nn.functional.normalize(torch.randn(F, H, S, 128, generator=g), dim=-1)
    beta = torch.rand(F, H, S, generator=g)
    A = torch.matmul((k * beta.unsqueeze(-1)).transpose(-1, -2), k)
    A = (0.5 * (A + A.transpose(-1, -2))).cuda()
    B = torch.randn(F, H, 128, 128, generator=g).cuda()
    alpha = (torch.rand(F, H, 128, generator=g) * 0.5 + 0.45).cuda()
    up = [torch.randn(F, H, 128, 128, generator=g).cuda() for _ in range(2)]

    def sym(fn):
        return lambda a, A_, B_: fn(a, 0.5 * (A_ + A_.transpose(-1, -2)), B_)

    outs, grads = _grads(sym(lambda a, A_, B_: lbg.vdn_factor(backend, a, A_, B_)),
                         (alpha, A, B), up)
    check_device_error()
    ref_outs, ref_grads = _grads(sym(backend.factor_apply), (alpha, A, B), up)
    for a, b in zip(outs, ref_outs):
        assert _rel(a, b) < 1e-4
    for a, b in zip(grads, ref_grads):
        assert _rel(a, b) < 1e-3


def test_branch_training_body_kernels_vs_pytorch():
    """The whole differentiable branch (conv features, statistics, factor, scans, gather,
    readout) with the kernels on vs off: same loss, same parameter gradients."""
    from vdn_minimax_h3_b200.models.linear_branch import BidirectionalLinearBranch
    from vdn_minimax_h3_b200.models.window import window_bounds
    torch.manual_seed(0)
    hidden, H, d, F, gh, gw = 256, 2, 128, 8, 4, 6
    S = gh * gw
    br = BidirectionalLinearBranch(hidden, H, d, delta_rule="vdn_solve",
                                   short_conv=("k", "v")).cuda()
    bounds = window_bounds(F, 1, chunk=2)
    g = torch.Generator().manual_seed(1)
    xv = torch.randn(F * S, hidden, generator=g).cuda()
    qkv = tuple(torch.randn(F * S, H, d, generator=g).cuda() for _ in range(3))
    text_x = torch.randn(10, hidden, generator=g).cuda()
    text_qkv = tuple(torch.randn(10, H, d, generator=g).cuda() for _ in range(3))
    up = torch.randn(F * S, H * d, generator=g).cuda()

    def run(kernels):
        lbg.USE_KERNELS = kernels
        try:
            br.zero_grad(set_to_none=True)
            out = br(xv, F, S, bounds, qkv, frame_size=(gh, gw), text_x=text_x,
                     text_qkv_raw=text_qkv)
            (out * up).sum().backward()
        finally:
            lbg.USE_KERNELS = True
        return out.detach(), {n: p.grad.detach().clone() for n, p in br.named_parameters()
                              if p.grad is not None}

    out_k, grads_k = run(True)
    check_device_error()
    out_r, grads_r = run(False)
    assert _rel(out_k, out_r) < 1e-3
    assert grads_k.keys() == grads_r.keys() and grads_k
    for name in grads_r:
        assert _rel(grads_k[name], grads_r[name]) < 2e-3, name


@pytest.mark.parametrize("F,gh,gw,H,l2", [(6, 5, 7, 2, True), (6, 5, 7, 2, False),
                                          (3, 24, 42, 1, True), (1, 4, 4, 1, True)])
def test_conv_features_backward_kernels(F, gh, gw, H, l2):
    """Short conv forward (two-pass kernels) and backward (conv_bwd.cu) vs fp32 autograd
    through the eager conv: output, input gradient and both weight gradients."""
    from vdn_minimax_h3_b200.models.linear_branch import conv_features_reference
    g = torch.Generator().manual_seed(F * 1000 + gh * 10 + gw)
    C = H * 128
    N = F * gh * gw
    tokens = torch.randn(N, H, 128, generator=g).to(torch.bfloat16).cuda()
    w_sp = (torch.randn(C, 5, 5, generator=g) * 0.2).cuda()
    w_tm = (torch.randn(C, 5, generator=g) * 0.45).cuda()
    up = torch.randn(N, H, 128, generator=g).to(torch.bfloat16).cuda()
    assert lbg.conv_kernel_ok(tokens, (gh, gw))
    x = tokens.clone().requires_grad_()
    ws, wt = w_sp.clone().requires_grad_(), w_tm.clone().requires_grad_()
    out = lbg.conv_features(x, ws, wt, F, (gh, gw), l2)
    (out.float() * up.float()).sum().backward()
    check_device_error()
    xr = tokens.float().requires_grad_()
    wsr, wtr = w_sp.clone().requires_grad_(), w_tm.clone().requires_grad_()
    ref = conv_features_reference(xr, wsr, wtr, F, (gh, gw), l2)
    (ref * up.float()).sum().backward()
    assert out.dtype == torch.bfloat16 and x.grad.dtype == torch.bfloat16
    assert _rel(out, ref) < 1e-2
    assert _rel(x.grad, xr.grad) < 2e-2
    assert _rel(ws.grad, wsr.grad) < 2e-2
    assert _rel(wt.grad, wtr.grad) < 2e-2
