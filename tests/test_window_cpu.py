"""Window softmax on CPU: the segment-wise training path (one attention per plan segment over
contiguous K/V slices) against the per-frame oracle, values and gradients."""
import pytest
import torch

from vdn_minimax_h3_b200.models.layout import SequenceLayout
from vdn_minimax_h3_b200.models.window import (window_bounds, window_softmax_reference,
                                               window_softmax_segments)


def _layout(text, audio, F, S):
    return SequenceLayout(seq_len=text + audio + F * S, video_start=text + audio, num_frames=F,
                          tokens_per_frame=S, frame_height=1, frame_width=S, text_start=0,
                          text_len=text)


@pytest.mark.parametrize("text,audio,F,S,H,chunk,radius,anchors", [
    (8, 6, 12, 10, 2, 2, 1, "both"),
    (8, 0, 9, 12, 3, 0, 1, "none"),
    (5, 3, 20, 6, 1, 5, 1, "both"),
    (7, 2, 10, 8, 2, 5, 1, "columns"),
    (7, 2, 10, 8, 2, 0, 2, "rows"),
    (4, 4, 3, 8, 2, 0, 5, "none"),            # the window covers every frame
])
def test_segments_match_per_frame_oracle(text, audio, F, S, H, chunk, radius, anchors):
    torch.manual_seed(0)
    lay = _layout(text, audio, F, S)
    bounds = window_bounds(F, radius, chunk)
    T, d = lay.seq_len, 16
    q, k, v = (torch.randn(T, H, d, dtype=torch.float64) for _ in range(3))
    up = torch.randn(T, H, d, dtype=torch.float64)

    def run(fn):
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        out = fn(*leaves, lay, bounds, d ** -0.5, anchors)
        (out * up).sum().backward()
        return out.detach(), [t.grad for t in leaves]

    out, grads = run(window_softmax_segments)
    ref, ref_grads = run(window_softmax_reference)
    torch.testing.assert_close(out, ref, rtol=1e-10, atol=1e-10)
    for a, b in zip(grads, ref_grads):
        torch.testing.assert_close(a, b, rtol=1e-9, atol=1e-10)
