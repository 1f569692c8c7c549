"""The linear branch's inference stages.

Each function is one stage of the forward-only body
(models/linear_branch.py: BidirectionalLinearBranch._readout_inference). On CUDA tensors a
stage runs its sm_100a kernel from csrc/linear_branch.cu; on CPU it runs the fp32 PyTorch
oracle the kernel is tested against (reference src/models/linear_attention/{features,scan,
delta_rule,kernels}.py).
"""
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.models import scan as scan_ref
from vdn_minimax_h3_b200.models.delta_rule import SanaDelta, VdnDelta
from vdn_minimax_h3_b200.models.linear_branch import activate as activate_ref
from vdn_minimax_h3_b200.models.linear_branch import conv_features_reference
from vdn_minimax_h3_b200.ops._ext import error_word, ext


def _native(t):
    return t.is_cuda


# ---------------------------------------------------------------------------- features
def activate(tokens, l2norm):
    """SiLU [+ L2 over d]: [N, H, d] -> same shape, same dtype."""
    if not _native(tokens):
        return activate_ref(tokens, l2norm)
    out = torch.empty(tokens.shape, dtype=tokens.dtype, device=tokens.device)
    ext().lb_activate(tokens, out, bool(l2norm))
    return out


# The short conv runs as two kernels (5x5 spatial into a bf16 intermediate, then 5-tap
# temporal + SiLU [+ L2]) unless this is False (one fused kernel, slower).
CONV_TWO_PASS = True


def conv_features(tokens, w_sp, w_tm, num_frames, frame_size, l2norm, two_pass=None):
    """5x5 depthwise spatial conv, 5-tap temporal conv, SiLU [, L2]."""
    if not _native(tokens):
        return conv_features_reference(tokens, w_sp, w_tm, num_frames, frame_size, l2norm)
    gh, gw = frame_size
    out = torch.empty(tokens.shape, dtype=tokens.dtype, device=tokens.device)
    tmp = None
    w_spatial = w_sp.float().reshape(-1, 25)
    if CONV_TWO_PASS if two_pass is None else two_pass:
        tmp = torch.empty(tokens.shape, dtype=tokens.dtype, device=tokens.device)
        w_spatial = w_spatial.t()           # the two-pass kernel reads taps [25, C]
    ext().lb_conv_features(tokens, w_spatial.contiguous().reshape(-1),
                           w_tm.float().reshape(-1).contiguous(), out, num_frames, gh, gw,
                           bool(l2norm), error_word(tokens.device), tmp)
    return out


# -------------------------------------------------------------------------- statistics
def frame_statistics(k, v, beta, a_fp32=True):
    """k, v [F, S, n, d] (token-major views of the projections); beta [F, S, n].
    -> A [F, n, d, d] fp32 symmetric, B [F, n, d, d] fp32."""
    if not _native(k):
        return scan_ref.frame_statistics(k.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3),
                                         beta.permute(0, 2, 1), a_fp32=a_fp32)
    Fr, S, n, d = k.shape
    A = torch.empty(Fr, n, d, d, dtype=torch.float32, device=k.device)
    B = torch.empty_like(A)
    ext().lb_frame_stats(k, v, beta.float().reshape(-1).contiguous(), A, B, error_word(k.device))
    return A, B


def factor_apply(backend, alpha, A, B):
    """transition = diag(alpha) * M^-1 (row scale), injection = (b B) M^-1 for the vdn
    rules; the sana rule is elementwise."""
    if not _native(A) or isinstance(backend, SanaDelta):
        return backend.factor_apply(alpha, A, B)
    assert isinstance(backend, VdnDelta)
    trans = torch.empty_like(A)
    inj = torch.empty_like(B)
    ext().lb_spd_factor(A.contiguous(), B.float().contiguous(), alpha.float().contiguous(), trans,
                        inj, float(backend.a_scale), float(backend.b_scale), error_word(A.device))
    return trans, inj


def run_scans(trans, inj, text_state=None):
    """prefix/suffix banks of the two serial recurrences. [F, n, d, d] fp32."""
    if not _native(trans):
        return scan_ref.run_scans(trans, inj, text_state)
    prefix = torch.empty_like(inj)
    suffix = torch.empty_like(inj)
    start = None if text_state is None else text_state.float().contiguous()
    ext().lb_scan(trans.contiguous(), inj.contiguous(), start, prefix, suffix, error_word(trans.device))
    return prefix, suffix


_GATHER_IDX = {}


def _gather_index_tables(bounds, num_frames, device):
    """The window-complement index tables of a layout, built once per (bounds, F, device):
    building them from Python lists is a pageable host-to-device copy, which would make
    the host wait for the stream on every layer."""
    key = (tuple(tuple(b) for b in bounds), num_frames, str(device))
    hit = _GATHER_IDX.get(key)
    if hit is None:
        idx = scan_ref.gather_indices(bounds, num_frames, device)
        table = torch.stack([idx["before_idx"], idx["after_idx"], idx["has_before"].long(),
                             idx["has_after"].long()], dim=1).to(torch.int32).contiguous()
        hit = _GATHER_IDX[key] = (idx, table)
    return hit


def gather_tables(alpha, bounds, bridge):
    """Per-frame gather indices [F, 4] (before, after, has_before, has_after) and the bridge
    factors prod(alpha) over the skipped frames, [F, H, d] each (fp32, from log-prefix sums)."""
    F_ = alpha.shape[0]
    idx, table = _gather_index_tables(bounds, F_, alpha.device)
    if bridge == "alpha":
        log_a = torch.log(alpha.float().clamp_min(1e-12))
        pre = torch.cat([torch.zeros_like(log_a[:1]), log_a.cumsum(0)])
        fr = idx["frames"]
        ab = torch.exp(pre[fr + 1] - pre[idx["bridge_before"]])
        aa = torch.exp(pre[idx["bridge_after"]] - pre[fr])
    else:
        ab = torch.ones_like(alpha, dtype=torch.float32)
        aa = torch.ones_like(alpha, dtype=torch.float32)
    return table, ab.contiguous(), aa.contiguous()


def gather(prefix, suffix, alpha, bounds, bridge, text_state, out_dtype=torch.bfloat16):
    """The complement of each frame's window, bridged into the frame. [F, n, d, d]."""
    if not _native(prefix):
        return scan_ref.gather_linear_state(prefix, suffix, alpha, bounds, bridge=bridge,
                                            text_state=text_state, out_dtype=out_dtype)
    table, ab, aa = gather_tables(alpha, bounds, bridge)
    out = torch.empty(prefix.shape, dtype=torch.bfloat16, device=prefix.device)
    start = None if text_state is None else text_state.float().contiguous()
    ext().lb_gather(prefix.contiguous(), suffix.contiguous(), table, ab, aa, start, out)
    return out if out_dtype in (None, torch.bfloat16) else out.to(out_dtype)


# --------------------------------------------------------------------------- readout
def readout_reference(q, state, norm_w, gate, eps, gate_logits=False):
    Fr, S, n, d = q.shape
    if gate_logits:
        gate = torch.sigmoid(gate.float())
    r = torch.einsum("fhvk,fshk->fshv", state.float(), q.float())
    ms = r.pow(2).mean(-1, keepdim=True)
    r = r * torch.rsqrt(ms + eps) * norm_w.float()
    return (r.reshape(Fr * S, n, d) * gate.float()).reshape(Fr * S, n * d).to(q.dtype)


def readout(q, state, norm_w, gate, eps, out=None, gate_logits=False, scatter=None):
    """RMSNorm(q . state^T) * w * gate, token-major [F*S, n*d]. `out` may be a strided view
    (the right half of the O-projection input). With gate_logits the gate is sigmoid(gate).
    scatter = (bases, row0, rows_per_rank): rows go to their Ulysses owners (see
    ops.attention.window_attention)."""
    if scatter is not None and not _native(q):
        raise ValueError("row-owner scatter needs the CUDA kernels")
    if not _native(q):
        r = readout_reference(q, state, norm_w, gate, eps, gate_logits)
        if out is not None:
            out.copy_(r)
            return out
        return r
    Fr, S, n, d = q.shape
    if out is None:
        out = torch.empty(Fr * S, n * d, dtype=q.dtype, device=q.device)
    bases, row0, rows = scatter if scatter is not None else ([], 0, 0)
    ext().lb_readout(q, state.contiguous(), norm_w.float().contiguous(), gate, out, float(eps),
                     bool(gate_logits), error_word(q.device), list(bases), int(row0), int(rows))
    return out


def text_state(branch, text_raw, text_beta):
    """TEXT_STATE_SCALE * S_text for a head range: the prompt written into a zero state as one
    delta-rule chunk of L rows (reference branch.py:178-216). text_raw = (q, k, v) [L, n, d]
    views; text_beta [L, n] fp32. [n, d, d] fp32."""
    q, k, v = text_raw
    L, n, d = k.shape
    kf = activate(k, True)
    vf = activate(v, False)
    A, B = frame_statistics(kf.view(1, L, n, d), vf.view(1, L, n, d), text_beta.reshape(1, L, n),
                            a_fp32=branch.a_fp32)
    ones = torch.ones(1, n, d, device=A.device, dtype=torch.float32)
    _, inj = factor_apply(branch.backend(L), ones, A, B)
    return branch.TEXT_STATE_SCALE * inj[0]


def bench_linear(timed, frames=100, heads=56):  # pragma: no cover - GPU tool
    """Each linear-branch stage at the full geometry: 100 inner frames x 1008 tokens x 56
    heads (anchors both); `heads` < 56 is one rank's share under sequence parallelism."""
    import json
    from vdn_minimax_h3_b200.models.delta_rule import VdnDelta
    from vdn_minimax_h3_b200.models.window import window_bounds
    Fr, S, n, d, gh, gw = frames, 1008, heads, 128, 24, 42
    dev = "cuda"
    raw = torch.randn(Fr * S, 3 * n * d + 8, device=dev, dtype=torch.bfloat16)
    q_raw = raw[:, :n * d].view(-1, n, d)
    k_raw = raw[:, n * d:2 * n * d].view(-1, n, d)
    w_sp = torch.randn(n * d, 5, 5, device=dev) / 5
    w_tm = torch.randn(n * d, 5, device=dev) / 2
    res = {}
    res["activate_q"] = timed(lambda: activate(q_raw, True))
    res["conv_features_k"] = timed(lambda: conv_features(k_raw, w_sp, w_tm, Fr, (gh, gw), True))
    res["conv_features_k_fused"] = timed(
        lambda: conv_features(k_raw, w_sp, w_tm, Fr, (gh, gw), True, two_pass=False))
    kf = conv_features(k_raw, w_sp, w_tm, Fr, (gh, gw), True)
    vf = conv_features(k_raw, w_sp, w_tm, Fr, (gh, gw), False)
    beta = torch.rand(Fr, S, n, device=dev)
    res["frame_stats"] = timed(lambda: frame_statistics(kf.view(Fr, S, n, d), vf.view(Fr, S, n, d), beta))
    A, B = frame_statistics(kf.view(Fr, S, n, d), vf.view(Fr, S, n, d), beta)
    alpha = torch.rand(Fr, n, d, device=dev) * 0.5 + 0.5
    res["spd_factor"] = timed(lambda: factor_apply(VdnDelta(S), alpha, A, B))
    trans, inj = factor_apply(VdnDelta(S), alpha, A, B)
    trans = trans * 0.05
    res["scan"] = timed(lambda: run_scans(trans, inj, None))
    pre, suf = run_scans(trans, inj, None)
    bounds = [(lo - 1, hi - 1) for lo, hi in window_bounds(Fr + 2, 1, 5)[1:-1]]
    res["gather"] = timed(lambda: gather(pre, suf, alpha, bounds, "alpha", None))
    state = gather(pre, suf, alpha, bounds, "alpha", None)
    qf = activate(q_raw, True)
    gate = torch.randn(Fr * S, n, d, device=dev, dtype=torch.bfloat16)
    w = torch.ones(d, device=dev)
    out = torch.empty(Fr * S, n * d, device=dev, dtype=torch.bfloat16)
    res["readout"] = timed(lambda: readout(qf.view(Fr, S, n, d), state, w, gate, 1e-6, out=out,
                                           gate_logits=True))
    print(json.dumps({"heads": n, "linear_branch_ms": {k: round(v, 3) for k, v in res.items()}}),
          flush=True)
