"""AdaLN-modulated RMSNorm and QK-norm + 3D RoPE.

Reference parity: `_pre_ref` (src/models/ops/fused_block.py:41-44: RMSNorm(x) *
(1 + scale[idx]) + shift[idx]) and `_qk_prep_body` (softmax_attention/kernels.py:27-30:
per-head RMSNorm then rotate-half RoPE). CUDA tensors run csrc/norm.cu; CPU tensors the
fp32 oracle below.
"""
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops._ext import ext


def adaln_rmsnorm_reference(x, weight, eps, table, shift_col, scale_col, idx):
    D = x.shape[-1]
    n = F.rms_norm(x.float(), (D,), None if weight is None else weight.float(), eps)
    tab = table.float()
    shift = tab[:, shift_col:shift_col + D].index_select(0, idx.long())
    scale = tab[:, scale_col:scale_col + D].index_select(0, idx.long())
    return (n * (1.0 + scale) + shift).to(x.dtype)


def adaln_rmsnorm(x, weight, eps, table, shift_col, scale_col, idx, out=None, fp8_out=None):
    """out = RMSNorm(x) * w * (1 + table[idx, scale]) + table[idx, shift]; [T, D] bf16.

    fp8_out = (q [T, D] uint8, sf) additionally (or, with out=False, only) writes the E4M3
    copy with one power-of-two scale per 1x128 block (ops.fp8 layout) for an fp8 GEMM."""
    if not x.is_cuda and fp8_out is not None:
        from vdn_minimax_h3_b200.ops import fp8
        y = adaln_rmsnorm_reference(x, weight, eps, table, shift_col, scale_col, idx)
        q, sf = fp8.quantize_act(y.to(torch.bfloat16))
        fp8_out[0].copy_(q)
        fp8_out[1].copy_(sf)
        if out is False:
            return fp8_out
        if out is not None:
            out.copy_(y)
            return out
        return y
    if not x.is_cuda:
        y = adaln_rmsnorm_reference(x, weight, eps, table, shift_col, scale_col, idx)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty_like(x)
    w = None if weight is None else weight.float().contiguous()
    q, sf = fp8_out if fp8_out is not None else (None, None)
    ext().adaln_rmsnorm(x, w, float(eps), table, int(shift_col), int(scale_col), idx,
                        None if out is False else out, q, sf)
    return fp8_out if out is False else out


def frame_sums(rows, num_frames, tokens_per_frame, row0=0, video_start=0, peers=None,
               slot_offset=0, out=None):
    """fp32 [F, D] per-frame column sums of the video rows found in `rows`.

    rows[0] is packed row `row0`; frame f spans packed rows [video_start + f*S, ... + S).
    A shard that holds part of a frame contributes its part (sum the shards' results).
    With `peers` (CUDA only: addresses of fp32 arrays, e.g. the ranks' copies of a
    symmetric-memory buffer) the sums are stored at peers[p] + slot_offset instead, only
    for the frames this shard touches; `out` is then not written."""
    F_, S = num_frames, tokens_per_frame
    if not rows.is_cuda:
        out = torch.zeros(F_, rows.shape[1], dtype=torch.float32)
        for f in range(F_):
            a = max(video_start + f * S, row0) - row0
            b = min(video_start + (f + 1) * S, row0 + rows.shape[0]) - row0
            if b > a:
                out[f] = rows[a:b].float().sum(0)
        return out
    if out is None:
        out = torch.empty(F_, rows.shape[1], dtype=torch.float32, device=rows.device)
    ext().frame_sums(rows, int(row0), int(video_start), int(F_), int(S), out,
                     [int(a) for a in (peers or [])], int(slot_offset))
    return out


def qk_prep_reference(src, heads, weight, eps, cos, sin):
    T = src.shape[0]
    d = src.shape[1] // heads
    t = F.rms_norm(src.float().view(T, heads, d), (d,), weight.float(), eps)
    rot = cos.shape[-1]
    x_rot, x_pass = t[..., :rot], t[..., rot:]
    x1, x2 = x_rot.chunk(2, dim=-1)
    rotated = torch.cat((-x2, x1), dim=-1)
    c, s = cos.float()[:, None, :], sin.float()[:, None, :]
    out = torch.cat((x_rot * c + rotated * s, x_pass), dim=-1)
    return out.reshape(T, heads * d).to(src.dtype)


def qk_prep(src, heads, weight, eps, cos, sin, out=None):
    """Per-head RMSNorm (weight [d]) then rotate-half RoPE. src [T, H*d] (row stride
    allowed) -> contiguous [T, H*d]."""
    if not src.is_cuda:
        y = qk_prep_reference(src, heads, weight, eps, cos, sin)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(src.shape[0], src.shape[1], dtype=src.dtype, device=src.device)
    ext().qk_prep(src, int(heads), weight.float().contiguous(), float(eps), cos, sin, out)
    return out
