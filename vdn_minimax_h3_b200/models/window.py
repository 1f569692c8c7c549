"""Window geometry for the softmax branch, the CPU oracle, and the attention work plan the
sm_100a window-attention kernel consumes.

Reference parity:
  * window_bounds: src/models/softmax_attention/window.py:26-52 (frame mode |dt| <= r;
    chunk-aligned "c<r>" mode, the window is a property of the K-frame chunk).
  * window_softmax_reference: window.py:56-111 (one dense attention per query frame;
    globals dense both ways; anchor rows/columns). It is the correctness oracle;
    window_softmax_segments computes the same attention per plan segment for training.
  * AttentionPlan replaces the reference's decomposed path (decomposed.py:108-221, a
    cuDNN dense leg plus FA4 varlen over GATHERED K/V) and its flex BlockMask: the c1 mask
    is a union of dense rectangles, so every query group's kept K/V set is a handful of
    CONTIGUOUS row ranges of the packed sequence. The kernel walks those ranges in place:
    no K/V gather, no mask tensor.
"""
from dataclasses import dataclass
from typing import List, Tuple

import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.models.layout import SequenceLayout

ANCHOR_FRAME_MODES = ("none", "columns", "rows", "both")
MAX_KV_RANGES = 4


def window_bounds(num_frames, radius, chunk=0):
    """Per-frame inclusive window [lo, hi], unclamped (frame or chunk-aligned mode)."""
    if chunk <= 0:
        return [(t - radius, t + radius) for t in range(num_frames)]
    return [(((t // chunk) - radius) * chunk, ((t // chunk) + radius + 1) * chunk - 1)
            for t in range(num_frames)]


def full_cover(bounds, num_frames):
    return all(lo <= 0 and hi >= num_frames - 1 for lo, hi in bounds)


def _sdpa_rows(q, k, v, scale):
    out = F.scaled_dot_product_attention(q.permute(1, 0, 2).unsqueeze(0),
                                         k.permute(1, 0, 2).unsqueeze(0),
                                         v.permute(1, 0, 2).unsqueeze(0), scale=scale)
    return out.squeeze(0).permute(1, 0, 2)


def window_softmax_reference(query, key, value, layout: SequenceLayout, bounds, scale,
                             anchor_frames="none"):
    """Exact window softmax: video x video pairs restricted to each frame's window, every
    pair touching a global row dense. [T, H, d] in and out."""
    heads, head_dim = query.shape[1], query.shape[2]
    vs, ve = layout.video_start, layout.video_end
    F_, S = layout.num_frames, layout.tokens_per_frame
    gidx = layout.global_index(query.device)
    out = torch.empty_like(query)
    if gidx.numel():
        out[gidx] = _sdpa_rows(query[gidx], key, value, scale)
    gk, gv = key[gidx], value[gidx]
    shape = (F_, S, heads, head_dim)
    vq, vk, vv = (t[vs:ve].view(shape) for t in (query, key, value))
    for f in range(F_):
        lo, hi = max(bounds[f][0], 0), min(bounds[f][1], F_ - 1)
        if anchor_frames in ("rows", "both") and f in (0, F_ - 1):
            lo, hi = 0, F_ - 1
        extra = [a for a in ((0, F_ - 1) if anchor_frames in ("columns", "both") else ())
                 if not lo <= a <= hi]
        extra = sorted(set(extra))
        ks = torch.cat([gk, vk[lo:hi + 1].reshape(-1, heads, head_dim)]
                       + [vk[a] for a in extra])
        vals = torch.cat([gv, vv[lo:hi + 1].reshape(-1, heads, head_dim)]
                         + [vv[a] for a in extra])
        out[vs + f * S: vs + (f + 1) * S] = _sdpa_rows(vq[f], ks, vals, scale)
    return out


def window_softmax_segments(query, key, value, layout: SequenceLayout, bounds, scale,
                            anchor_frames="none"):
    """The same attention as `window_softmax_reference`, one dense attention per plan
    segment (`plan_segments`: consecutive query frames sharing a window, plus the dense
    global / anchor rows) over that segment's <= MAX_KV_RANGES contiguous K/V row slices.
    The differentiable training path: under the c1 window 81 frames are 17 segments, so
    there are ~5x fewer attention calls and K/V copies than per frame. [T, H, d]."""
    segs = sorted(plan_segments(layout, bounds, anchor_frames), key=lambda s: s.q_start)
    outs = []
    for seg in segs:
        if len(seg.kv) == 1:
            a, b = seg.kv[0]
            ks, vals = key[a:b], value[a:b]
        else:
            ks = torch.cat([key[a:b] for a, b in seg.kv])
            vals = torch.cat([value[a:b] for a, b in seg.kv])
        outs.append(_sdpa_rows(query[seg.q_start:seg.q_end], ks, vals, scale))
    return outs[0] if len(outs) == 1 else torch.cat(outs)


@dataclass
class Segment:
    """A contiguous run of query rows sharing one K/V set (<= MAX_KV_RANGES ranges)."""
    q_start: int
    q_end: int
    kv: List[Tuple[int, int]]


def _merge(ranges):
    out = []
    for a, b in sorted(r for r in ranges if r[0] < r[1]):
        if out and out[-1][1] >= a:
            out[-1] = (out[-1][0], max(out[-1][1], b))
        else:
            out.append((a, b))
    return out


def plan_segments(layout: SequenceLayout, bounds, anchor_frames="none", dense=False):
    """Query segments and their K/V row ranges for the window mask.

    dense=True (a window covering all frames) is one segment over everything."""
    T = layout.seq_len
    if dense or full_cover(bounds, layout.num_frames):
        return [Segment(0, T, [(0, T)])]
    F_, S, vs = layout.num_frames, layout.tokens_per_frame, layout.video_start
    anchors = {0, F_ - 1} if anchor_frames in ("columns", "rows", "both") else set()
    dense_rows = anchors if anchor_frames in ("rows", "both") else set()
    dense_cols = anchors if anchor_frames in ("columns", "both") else set()
    globals_ = layout.global_ranges()

    def frame_rows(f):
        return (vs + f * S, vs + (f + 1) * S)

    segs = []
    for a, b in _merge(globals_ + [frame_rows(f) for f in sorted(dense_rows)]):
        segs.append(Segment(a, b, [(0, T)]))
    groups = []
    for f in range(F_):
        if f in dense_rows:
            continue
        if groups and groups[-1][-1] == f - 1 and bounds[groups[-1][-1]] == bounds[f]:
            groups[-1].append(f)
        else:
            groups.append([f])
    for frames in groups:
        lo, hi = bounds[frames[0]]
        lo, hi = max(lo, 0), min(hi, F_ - 1)
        kv_frames = set(range(lo, hi + 1)) | dense_cols
        kv = _merge(globals_ + [frame_rows(f) for f in kv_frames])
        if len(kv) > MAX_KV_RANGES:
            raise ValueError(f"window needs {len(kv)} K/V ranges > {MAX_KV_RANGES}")
        segs.append(Segment(frame_rows(frames[0])[0], frame_rows(frames[-1])[1], kv))
    covered = sum(s.q_end - s.q_start for s in segs)
    if covered != T:
        raise ValueError(f"plan covers {covered} of {T} rows")
    return segs


class AttentionPlan:
    """Device tables for the window-attention kernel, built once per (layout, bounds).

    tiles:  int32 [n_tiles, 4]  (q_start, q_end, segment, kv_rows) for each work item of up
            to `block_q` (256) query rows -- the kernel runs it as two 128-row tiles sharing
            every K/V block -- longest K/V first so the persistent schedule ends balanced.
    kv:     int32 [n_segments, 2 * MAX_KV_RANGES] (start, end) pairs, empty ranges (0, 0).
    """

    def __init__(self, layout, bounds, anchor_frames="none", device="cpu", block_q=256,
                 dense=False, segments=None):
        self.segments = (segments if segments is not None
                         else plan_segments(layout, bounds, anchor_frames, dense=dense))
        kv = torch.zeros(len(self.segments), 2 * MAX_KV_RANGES, dtype=torch.int32)
        tiles, cost = [], []
        for i, seg in enumerate(self.segments):
            for j, (a, b) in enumerate(seg.kv):
                kv[i, 2 * j], kv[i, 2 * j + 1] = a, b
            kv_len = sum(b - a for a, b in seg.kv)
            for q0 in range(seg.q_start, seg.q_end, block_q):
                tiles.append((q0, min(q0 + block_q, seg.q_end), i, kv_len))
                cost.append(kv_len)
        order = sorted(range(len(tiles)), key=lambda t: -cost[t])
        self.tiles = torch.tensor([tiles[t] for t in order], dtype=torch.int32).view(-1, 4).to(device)
        self.kv = kv.to(device)
        self.num_tiles = len(tiles)
        self.kv_rows_total = sum((t[1] - t[0]) * t[3] for t in tiles)

    @classmethod
    def dense_rows(cls, T, device="cpu", block_q=256):
        """Every row attends to every row (the dense teacher) -- no layout needed."""
        return cls(None, None, device=device, block_q=block_q, segments=[Segment(0, T, [(0, T)])])

    def flops(self, heads, head_dim):
        """Useful attention FLOPs (QK^T and PV) of the plan."""
        return 4.0 * self.kv_rows_total * heads * head_dim


def transpose_segments(segments: List[Segment]) -> List[Segment]:
    """The same attention pattern seen from the keys: for every maximal run of key rows
    attended by the same query rows, a Segment(k_start, k_end, query ranges) (the `kv`
    field then holds the <= MAX_KV_RANGES merged QUERY ranges)."""
    cuts = sorted({x for seg in segments for a, b in seg.kv for x in (a, b)})
    runs = []
    for lo, hi in zip(cuts[:-1], cuts[1:]):
        qs = _merge([(seg.q_start, seg.q_end) for seg in segments
                     if any(a <= lo and hi <= b for a, b in seg.kv)])
        if not qs:
            continue
        if runs and runs[-1].q_end == lo and runs[-1].kv == qs:
            runs[-1] = Segment(runs[-1].q_start, hi, qs)
        else:
            runs.append(Segment(lo, hi, qs))
    for r in runs:
        if len(r.kv) > MAX_KV_RANGES:
            raise ValueError(f"keys {r.q_start}:{r.q_end} are read by {len(r.kv)} query ranges "
                             f"> {MAX_KV_RANGES}")
    return runs


class TrainingAttentionPlan:
    """The three tables the training attention needs for one (layout, bounds): the forward
    plan (256-row items), the dq-pass plan (the same segments in 128-row query tiles) and
    the dk/dv-pass plan (128-row key tiles over the transposed segments)."""

    def __init__(self, segments: List[Segment], device):
        self.forward = AttentionPlan(None, None, device=device, segments=segments)
        self.dq = AttentionPlan(None, None, device=device, block_q=128, segments=segments)
        self.dkv = AttentionPlan(None, None, device=device, block_q=128,
                                 segments=transpose_segments(segments))

    @classmethod
    def for_layout(cls, layout, bounds, anchor_frames, device, dense=False):
        return cls(plan_segments(layout, bounds, anchor_frames, dense=dense), device)

    @classmethod
    def dense_rows(cls, T, device):
        return cls([Segment(0, T, [(0, T)])], device)
