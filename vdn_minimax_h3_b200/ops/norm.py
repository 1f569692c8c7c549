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


def adaln_rmsnorm(x, weight, eps, table, shift_col, scale_col, idx, out=None,
                  frame_sums=None, video_start=0, tokens_per_frame=1, num_frames=0):
    """out = RMSNorm(x) * w * (1 + table[idx, scale]) + table[idx, shift]; [T, D] bf16.

    With `frame_sums` (fp32 [F, D], zeroed by the caller) the kernel also accumulates the
    per-frame sums of the OUTPUT over the video rows -- the frame means the linear branch's
    alpha needs, without a second pass over the tensor."""
    if not x.is_cuda:
        y = adaln_rmsnorm_reference(x, weight, eps, table, shift_col, scale_col, idx)
        if frame_sums is not None and num_frames:
            vs = video_start
            frame_sums += y[vs:vs + num_frames * tokens_per_frame].float().view(
                num_frames, tokens_per_frame, -1).sum(1)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty_like(x)
    w = None if weight is None else weight.float().contiguous()
    ext().adaln_rmsnorm(x, w, float(eps), table, int(shift_col), int(scale_col), idx, out,
                        frame_sums, int(video_start), int(tokens_per_frame), int(num_frames))
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
