"""Differentiable window softmax attention on the sm_100a kernels, for training.

Forward: the inference kernel (csrc/attention.cu) over the plan, ungated, also writing each
row's log2-sum-exp. Backward: csrc/attention_bwd.cu -- a dq pass over the forward plan (one
CTA per 128 query rows: S, dP on tcgen05, dS in registers, dQ += dS K in TMEM, and
delta = rowsum(dO * O) on the way) then a dk/dv pass over the transposed plan (one CTA per
128 key rows: S^T, dP^T, dV += P^T dO, dK += dS^T Q). No mask tensor and no K/V gather in
either direction: the plans hold <= 4 contiguous row ranges per tile.

`window_attention_train` is what the hybrid block's softmax branch and the dense teacher
call for bf16 CUDA tensors with 128-wide heads; other inputs take the per-segment SDPA path
of models/window.py.

Reference parity: the training path of src/models/softmax_attention/flex_attention.py:
86-90, 177-210 (flex attention with a compiled block-sparse backward) and the dense SDPA of
the teacher; the gradients are the standard softmax-attention ones.
"""
import torch

from vdn_minimax_h3_b200.ops._ext import error_word, ext

HEAD_DIM = 128


class _WindowAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, plan, scale):
        T, H, d = q.shape
        out = torch.empty(T, H * d, dtype=q.dtype, device=q.device)
        lse = torch.empty(H, T, dtype=torch.float32, device=q.device)
        ext().window_attention(q, k, v, plan.forward.tiles, plan.forward.kv, None, out,
                               float(scale), error_word(q.device), [], 0, 0, None, lse)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.plan, ctx.scale = plan, float(scale)
        return out.view(T, H, d)

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        T, H, d = q.shape
        dout = dout.to(q.dtype).contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        delta = torch.empty(H, T, dtype=torch.float32, device=q.device)
        plan = ctx.plan
        ext().window_attention_bwd(q, k, v, out.view(T, H, d), dout, lse, delta, dq, dk, dv,
                                   plan.dq.tiles, plan.dq.kv, plan.dkv.tiles, plan.dkv.kv,
                                   ctx.scale, error_word(q.device))
        return dq, dk, dv, None, None


def kernel_path_ok(q, k, v):
    """bf16 CUDA [T, H, 128] with contiguous heads and 16-byte aligned rows."""
    for t in (q, k, v):
        if not (t.is_cuda and t.dtype == torch.bfloat16 and t.dim() == 3 and t.shape[2] == HEAD_DIM
                and t.stride(2) == 1 and t.stride(1) == HEAD_DIM and (t.stride(0) * 2) % 16 == 0
                and t.data_ptr() % 16 == 0):
            return False
    return True


def window_attention_train(q, k, v, plan, scale):
    """Softmax attention of q [T, H, 128] over the rows `plan` (a TrainingAttentionPlan)
    allows; returns [T, H, 128] and is differentiable in q, k and v. Without autograd the
    forward kernel runs alone (no log-sum-exp is kept)."""
    if not (torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad)):
        T, H, d = q.shape
        out = torch.empty(T, H * d, dtype=q.dtype, device=q.device)
        ext().window_attention(q, k, v, plan.forward.tiles, plan.forward.kv, None, out,
                               float(scale), error_word(q.device), [], 0, 0, None, None)
        return out.view(T, H, d)
    return _WindowAttention.apply(q, k, v, plan, scale)


ATTENTION_KERNELS = True       # module switch: False sends training attention to SDPA
_PLANS = {}


def _cached(key, build):
    plan = _PLANS.get(key)
    if plan is None:
        if len(_PLANS) > 32:
            _PLANS.clear()
        plan = _PLANS[key] = build()
    return plan


def window_plan(layout, bounds, anchor_frames, device, dense=False):
    """TrainingAttentionPlan of a hybrid block's softmax branch (shared by all blocks)."""
    from vdn_minimax_h3_b200.models.window import TrainingAttentionPlan
    key = ("window", layout, tuple(map(tuple, bounds)) if bounds is not None else None,
           anchor_frames, bool(dense), str(device))
    return _cached(key, lambda: TrainingAttentionPlan.for_layout(layout, bounds, anchor_frames,
                                                                 device, dense=dense))


def dense_plan(T, device):
    """TrainingAttentionPlan of T rows that all attend to each other (dense teacher)."""
    from vdn_minimax_h3_b200.models.window import TrainingAttentionPlan
    return _cached(("dense", int(T), str(device)), lambda: TrainingAttentionPlan.dense_rows(T, device))


def bench_attention_train(timed, frames=81, heads=56):  # pragma: no cover - GPU tool
    """Training attention at the Stage-B shape (81 latent frames, 56 heads, c1 window with
    anchors): forward + backward of the kernels against autograd of the per-segment SDPA
    path under cuDNN and flash, and the dense teacher forward against cuDNN SDPA. ms per
    layer; FLOPs counted as 4 * pairs * d (forward) and 2.5x that (backward)."""
    import json
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from vdn_minimax_h3_b200.models.layout import SequenceLayout
    from vdn_minimax_h3_b200.models.window import window_bounds, window_softmax_segments
    text, audio, S, d = 800, frames * 455 // 102, 1008, HEAD_DIM
    lay = SequenceLayout(seq_len=text + audio + frames * S, video_start=text + audio,
                         num_frames=frames, tokens_per_frame=S, frame_height=24, frame_width=42,
                         text_start=0, text_len=text)
    T = lay.seq_len
    bounds = window_bounds(frames, 1, 5)
    plan = window_plan(lay, bounds, "both", "cuda")
    fl = plan.forward.flops(heads, d)
    q, k, v = (torch.randn(T, heads, d, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    up = torch.randn_like(q)
    qg, kg, vg = (t.clone().requires_grad_() for t in (q, k, v))
    res = dict(case="attention_train_c1_both", T=T, heads=heads)

    def ours_fwd():
        with torch.no_grad():
            window_attention_train(q, k, v, plan, d ** -0.5)

    def ours_fb():
        window_attention_train(qg, kg, vg, plan, d ** -0.5).backward(up)

    res["ours_fwd_ms"] = timed(ours_fwd)
    res["ours_fwd_bwd_ms"] = timed(ours_fb)
    res["ours_bwd_ms"] = res["ours_fwd_bwd_ms"] - res["ours_fwd_ms"]
    res["ours_bwd_tflops"] = 2.5 * fl / res["ours_bwd_ms"] / 1e9
    for name, backend in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
        def lib_fb():
            with sdpa_kernel([backend]):
                window_softmax_segments(qg, kg, vg, lay, bounds, d ** -0.5, "both").backward(up)
        try:
            res[f"{name}_segments_fwd_bwd_ms"] = timed(lib_fb)
        except RuntimeError as e:
            res[f"{name}_error"] = str(e).splitlines()[0][:160]
    dplan = dense_plan(T, "cuda")
    dfl = dplan.forward.flops(heads, d)

    def dense_ours():
        with torch.no_grad():
            window_attention_train(q, k, v, dplan, d ** -0.5)

    res["dense_ours_ms"] = timed(dense_ours, iters=3, warmup=1)
    res["dense_ours_tflops"] = dfl / res["dense_ours_ms"] / 1e9
    qt, kt, vt = (t.transpose(0, 1)[None] for t in (q, k, v))
    for name, backend in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
        def dense_lib():
            with torch.no_grad(), sdpa_kernel([backend]):
                torch.nn.functional.scaled_dot_product_attention(qt, kt, vt, scale=d ** -0.5)
        try:
            res[f"dense_{name}_ms"] = timed(dense_lib, iters=3, warmup=1)
        except RuntimeError as e:
            res[f"dense_{name}_error"] = str(e).splitlines()[0][:160]
    print(json.dumps(res), flush=True)
    return res
