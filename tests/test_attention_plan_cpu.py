"""The training attention's plans on CPU: the transposed plan (key runs and the query ranges
that read them) covers exactly the (query, key) pairs of the forward plan, for window,
anchor and dense layouts."""
import itertools

import pytest

from vdn_minimax_h3_b200.models.layout import SequenceLayout
from vdn_minimax_h3_b200.models.window import (Segment, TrainingAttentionPlan, plan_segments,
                                               transpose_segments, window_bounds)


def _pairs(segments):
    return {(qi, ki) for s in segments for qi in range(s.q_start, s.q_end)
            for a, b in s.kv for ki in range(a, b)}


@pytest.mark.parametrize("chunk,radius,anchors", [(2, 1, "both"), (0, 1, "none"), (3, 0, "rows"),
                                                  (2, 0, "columns")])
def test_transposed_pairs_equal(chunk, radius, anchors):
    lay = SequenceLayout(seq_len=7 + 5 + 9 * 4, video_start=12, num_frames=9, tokens_per_frame=4,
                         text_start=0, text_len=7)
    segs = plan_segments(lay, window_bounds(9, radius, chunk), anchors)
    tr = transpose_segments(segs)
    assert {(q, k) for q, k in _pairs(segs)} == {(q, k) for k, q in _pairs(tr)}
    # key runs are disjoint and sorted
    for a, b in itertools.pairwise(tr):
        assert a.q_end <= b.q_start


def test_training_plan_tables():
    segs = [Segment(0, 300, [(0, 300)])]
    plan = TrainingAttentionPlan(segs, "cpu")
    assert plan.forward.num_tiles == 2 and plan.dq.num_tiles == 3 and plan.dkv.num_tiles == 3
    assert plan.dkv.kv[0, :2].tolist() == [0, 300]
