"""Window softmax attention over an AttentionPlan (models/window.py).

CUDA tensors run the sm_100a flash-attention kernel of csrc/attention.cu: tcgen05 MMAs for
S = Q K^T and O += P V with both accumulators in TMEM, Q/K/V tiles by TMA (no multicast),
online softmax in registers, K/V walked over the plan's contiguous row ranges in place (no
gather, no mask tensor), the per-head softmax gate applied in the epilogue. CPU tensors run
the dense-segment oracle below.

Reference parity: the window softmax of src/models/softmax_attention/{window,decomposed,
flex_attention}.py and the gate of kernels.py:51-67.
"""
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops._ext import error_word, ext


def window_attention_reference(q, k, v, plan, scale, gate_logits=None):
    """q, k, v [T, H, d]; returns [T, H*d] (gated when gate_logits [T, H] is given)."""
    T, H, d = q.shape
    out = torch.empty(T, H, d, dtype=torch.float32, device=q.device)
    for seg in plan.segments:
        kv_rows = torch.cat([torch.arange(a, b, device=q.device) for a, b in seg.kv])
        qs = q[seg.q_start:seg.q_end].float().transpose(0, 1)
        ks = k[kv_rows].float().transpose(0, 1)
        vs = v[kv_rows].float().transpose(0, 1)
        o = F.scaled_dot_product_attention(qs[None], ks[None], vs[None], scale=scale)[0]
        out[seg.q_start:seg.q_end] = o.transpose(0, 1)
    if gate_logits is not None:
        out = out * torch.sigmoid(gate_logits.float())[..., None]
    return out.reshape(T, H * d).to(q.dtype)


def window_attention(q, k, v, plan, scale, gate_logits=None, out=None, scatter=None, trace=None,
                     lse=None):
    """q, k, v: [T, H, d] views (row stride allowed, d contiguous). out: [T, H*d] view.

    scatter = (bases, row0, rows_per_rank) sends output row t to its Ulysses owner
    r = (row0 + t) // rows_per_rank instead: bases[r] is the address of that owner's
    destination at shard row 0 (this rank's first column), rows keep `out`'s row stride.
    lse: optional fp32 [H, T] receiving each row's log2-sum-exp (training forward)."""
    if scatter is not None and not q.is_cuda:
        raise ValueError("row-owner scatter needs CUDA tensors")
    if not q.is_cuda:
        y = window_attention_reference(q, k, v, plan, scale, gate_logits)
        if out is not None:
            out.copy_(y)
            return out
        return y
    T, H, d = q.shape
    if out is None:
        out = torch.empty(T, H * d, dtype=q.dtype, device=q.device)
    bases, row0, rows = scatter if scatter is not None else ([], 0, 0)
    ext().window_attention(q, k, v, plan.tiles, plan.kv, gate_logits, out, float(scale),
                           error_word(q.device), list(bases), int(row0), int(rows), trace, lse)
    return out


def bench_attention(timed, frames=102, heads=56):  # pragma: no cover - GPU tool
    import json
    from vdn_minimax_h3_b200.models.layout import SequenceLayout
    from vdn_minimax_h3_b200.models.window import AttentionPlan, window_bounds
    T_text, T_audio, Fr, S, H, d = 800, 1150, frames, 1008, heads, 128
    layout = SequenceLayout(seq_len=T_text + T_audio + Fr * S, video_start=T_text + T_audio,
                            num_frames=Fr, tokens_per_frame=S, frame_height=24, frame_width=42,
                            text_start=0, text_len=T_text)
    plan = AttentionPlan(layout, window_bounds(Fr, 1, 5), "both", device="cuda")
    T = layout.seq_len
    q = torch.randn(T, H, d, device="cuda", dtype=torch.bfloat16)
    k, v = torch.randn_like(q), torch.randn_like(q)
    fl = plan.flops(H, d)
    prev = ext().attention_variant()
    for var in range(8):
        ext().attention_set_variant(var)
        ms = timed(lambda: window_attention(q, k, v, plan, d ** -0.5))
        print(json.dumps(dict(case="window_attention_c1_both", T=T, heads=H, variant=var, ms=ms,
                              tflops=fl / ms / 1e9)), flush=True)
    ext().attention_set_variant(prev)


TRACE_EVENTS = ("s_wait", "s_ready", "ld_done", "max_done", "exp_done", "p_arrive")


def trace_attention(frames=102, heads=56, blocks=(8, 60), variant=None):  # pragma: no cover
    """Per-phase clock cycles of CTA 0's softmax / MMA pipeline (kernel timestamps) for one
    kernel variant (default: the current one). GPU tool."""
    import json
    from vdn_minimax_h3_b200.models.layout import SequenceLayout
    from vdn_minimax_h3_b200.models.window import AttentionPlan, window_bounds
    S = 1008
    lay = SequenceLayout(seq_len=1950 + frames * S, video_start=1950, num_frames=frames,
                         tokens_per_frame=S, frame_height=24, frame_width=42, text_start=0,
                         text_len=800)
    plan = AttentionPlan(lay, window_bounds(frames, 1, 5), "both", device="cuda")
    q = torch.randn(lay.seq_len, heads, 128, device="cuda", dtype=torch.bfloat16)
    k, v = torch.randn_like(q), torch.randn_like(q)
    tr = torch.zeros(12 * 64 + 4, dtype=torch.int64, device="cuda")
    prev = ext().attention_variant()
    if variant is not None:
        ext().attention_set_variant(variant)
    try:
        window_attention(q, k, v, plan, 128 ** -0.5)
        window_attention(q, k, v, plan, 128 ** -0.5, trace=tr)
        torch.cuda.synchronize()
    finally:
        ext().attention_set_variant(prev)
    stamps = tr[12 * 64:].cpu().double()
    t = tr[:12 * 64].view(6, 2, 64).cpu().double()
    a, b = blocks
    ev = {n: t[i] for i, n in enumerate(TRACE_EVENTS)}
    out = {}
    for tile in (0, 1):
        d = lambda x, y: float((ev[y][tile, a:b] - ev[x][tile, a:b]).mean())  # noqa: E731
        out[f"tile{tile}"] = {
            "wait_S": d("s_wait", "s_ready"), "tmem_load": d("s_ready", "ld_done"),
            "row_max": d("ld_done", "max_done"), "exp_pack_store": d("max_done", "exp_done"),
            "wait_st_arrive": d("exp_done", "p_arrive"),
            "P_arrive_to_next_S": float((ev["s_ready"][tile, a + 1:b + 1] - ev["p_arrive"][tile, a:b]).mean()),
            "block_period": float((ev["s_ready"][tile, a + 1:b + 1] - ev["s_ready"][tile, a:b]).mean()),
        }
    # timeline of a few blocks relative to tile 0's first S-ready: shows whether the two
    # tiles' softmax phases alternate or overlap
    t0 = ev["s_ready"][0, a]
    line = {}
    for n in ("s_ready", "max_done", "exp_done", "p_arrive"):
        line[n] = [[int(ev[n][tile, i] - t0) for i in range(a, a + 6)] for tile in (0, 1)]
    out["timeline"] = line
    out["sm_mhz"] = float((stamps[3] - stamps[1]) / (stamps[2] - stamps[0]) * 1e3)
    out["variant"] = ext().attention_variant() if variant is None else variant
    print(json.dumps({"attention_trace_cycles": out}), flush=True)
    return out


def bench_attention_vs_cudnn(timed, frames=102, heads=56):  # pragma: no cover - GPU tool
    """A/B of the window-attention kernel against cuDNN SDPA (and torch's flash backend) on
    the SAME work: the library runs one dense attention per plan segment over that
    segment's K/V rows, gathered and laid out [1, H, L, d] before timing (the gather is not
    charged to it). All numbers are ms per layer, 56 heads, the whole 14.4 s clip."""
    import json
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from vdn_minimax_h3_b200.models.layout import SequenceLayout
    from vdn_minimax_h3_b200.models.window import AttentionPlan, window_bounds
    T_text, T_audio, Fr, S, H, d = 800, 1150, frames, 1008, heads, 128
    layout = SequenceLayout(seq_len=T_text + T_audio + Fr * S, video_start=T_text + T_audio,
                            num_frames=Fr, tokens_per_frame=S, frame_height=24, frame_width=42,
                            text_start=0, text_len=T_text)
    plan = AttentionPlan(layout, window_bounds(Fr, 1, 5), "both", device="cuda")
    T = layout.seq_len
    q = torch.randn(T, H, d, device="cuda", dtype=torch.bfloat16)
    k, v = torch.randn_like(q), torch.randn_like(q)
    fl = plan.flops(H, d)
    ours = timed(lambda: window_attention(q, k, v, plan, d ** -0.5))
    segs = []
    for seg in plan.segments:
        rows = torch.cat([torch.arange(a, b, device="cuda") for a, b in seg.kv])
        segs.append((q[seg.q_start:seg.q_end].permute(1, 0, 2).unsqueeze(0).contiguous(),
                     k[rows].permute(1, 0, 2).unsqueeze(0).contiguous(),
                     v[rows].permute(1, 0, 2).unsqueeze(0).contiguous()))
    res = dict(case="window_attention_c1_both_ab", T=T, heads=H, segments=len(segs),
               variant=ext().attention_variant(), ours_ms=ours, ours_tflops=fl / ours / 1e9)
    for name, backend in (("cudnn", SDPBackend.CUDNN_ATTENTION),
                          ("flash", SDPBackend.FLASH_ATTENTION)):
        def run():
            with sdpa_kernel([backend]):
                for qs, ks, vs in segs:
                    F.scaled_dot_product_attention(qs, ks, vs, scale=d ** -0.5)
        try:
            ms = timed(run)
            res[f"{name}_ms"] = ms
            res[f"{name}_tflops"] = fl / ms / 1e9
        except RuntimeError as e:  # backend not available for this shape / GPU
            res[f"{name}_error"] = str(e).splitlines()[0][:200]
    print(json.dumps(res), flush=True)
    return res
