"""Training window attention on a B200: the sm_100a forward (with its log-sum-exp) and the
dq / dk-dv backward kernels against fp32 autograd through the per-frame SDPA oracle, for
window plans with global rows, anchors and ragged ranges, and for the dense plan."""
import pytest
import torch

from vdn_minimax_h3_b200.models.layout import SequenceLayout
from vdn_minimax_h3_b200.models.window import (TrainingAttentionPlan, plan_segments,
                                               transpose_segments, window_bounds,
                                               window_softmax_reference)
from vdn_minimax_h3_b200.ops import attention_grad as ag
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


def _layout(text, audio, F, S):
    return SequenceLayout(seq_len=text + audio + F * S, video_start=text + audio, num_frames=F,
                          tokens_per_frame=S, frame_height=1, frame_width=S, text_start=0,
                          text_len=text)


def _check(q, k, v, plan, oracle, scale):
    g = torch.Generator().manual_seed(1)
    up = torch.randn(q.shape, generator=g).to(torch.bfloat16).cuda()
    qk = [t.clone().requires_grad_() for t in (q, k, v)]
    out = ag.window_attention_train(*qk, plan, scale)
    out.backward(up)
    torch.cuda.synchronize()
    check_device_error()
    ref_in = [t.detach().float().cpu().requires_grad_() for t in (q, k, v)]
    ref = oracle(*ref_in)
    ref.backward(up.float().cpu())
    errs = [_rel(out.detach(), ref.detach())] + [_rel(a.grad, b.grad) for a, b in zip(qk, ref_in)]
    return errs


@pytest.mark.parametrize("text,audio,F,S,H,chunk,radius,anchors", [
    (40, 30, 12, 100, 2, 2, 1, "both"),
    (17, 5, 20, 60, 1, 5, 1, "both"),
    (64, 0, 9, 128, 2, 0, 1, "none"),
])
def test_window_attention_backward_matches_fp32_autograd(text, audio, F, S, H, chunk, radius, anchors):
    torch.manual_seed(0)
    lay = _layout(text, audio, F, S)
    bounds = window_bounds(F, radius, chunk)
    T = lay.seq_len
    q, k, v = (torch.randn(T, H, 128) * 1.5).to(torch.bfloat16).cuda(), \
        torch.randn(T, H, 128).to(torch.bfloat16).cuda(), torch.randn(T, H, 128).to(torch.bfloat16).cuda()
    plan = TrainingAttentionPlan.for_layout(lay, bounds, anchors, "cuda")
    scale = 128 ** -0.5
    errs = _check(q, k, v, plan,
                  lambda a, b, c: window_softmax_reference(a, b, c, lay, bounds, scale, anchors), scale)
    assert max(errs) < 2e-2, errs


@pytest.mark.parametrize("T,H", [(300, 2), (129, 1)])
def test_dense_attention_backward_matches_fp32_autograd(T, H):
    torch.manual_seed(1)
    q, k, v = (torch.randn(T, H, 128).to(torch.bfloat16).cuda() for _ in range(3))
    scale = 128 ** -0.5

    def dense(a, b, c):
        o = torch.nn.functional.scaled_dot_product_attention(
            a.transpose(0, 1)[None], b.transpose(0, 1)[None], c.transpose(0, 1)[None], scale=scale)
        return o[0].transpose(0, 1)

    errs = _check(q, k, v, ag.dense_plan(T, "cuda"), dense, scale)
    assert max(errs) < 2e-2, errs


def test_transposed_plan_covers_the_same_pairs():
    lay = _layout(40, 30, 12, 100)
    segs = plan_segments(lay, window_bounds(12, 1, 2), "both")
    pairs = lambda ss: sum((s.q_end - s.q_start) * sum(b - a for a, b in s.kv) for s in ss)  # noqa: E731
    assert pairs(transpose_segments(segs)) == pairs(segs)
