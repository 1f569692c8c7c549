"""Differentiable AdaLN-modulated RMSNorm for the training body of the DiT block:
y = RMSNorm(x) * w * (1 + scale[idx]) + shift[idx] (reference: the H3 block's norm1 / norm2
with the AdaLN modulation, src/models/ops/fused_block.py:41-44, differentiated there through
autograd of the eager ops).

Forward: the inference kernel `adaln_rmsnorm` (csrc/norm.cu; one read of x, one write, the
per-row modulation gathered in registers). Backward: `adaln_rmsnorm_bwd` (csrc/norm_bwd.cu)
for dx = r g - (r^3 / D) x sum(g x), g = dy * w * (1 + scale[idx]); the gradients of w, shift
and scale (all frozen in the shipped training stages) only when they are required, in
PyTorch. `adaln_modulated_norm` takes the kernels for every bf16 CUDA row set -- with or
without autograd -- and the eager expression otherwise.

The kernel keeps the normalisation and the affine chain in fp32 and rounds once, where the
eager expression rounds to bf16 after each op, so the two differ by up to about two bf16
ulps. The choice is therefore made by the module flag `NORM_KERNELS` and the tensors' dtype
and layout only, never by whether a graph is being recorded: a no-grad teacher forward and
the student forward it is compared with (Stage A2 / B losses, the DMD real score) always
run the same norm implementation, so no loss carries a difference between two norms.
"""
import torch

NORM_KERNELS = True
MAX_DIM = 12288          # widest row of the forward kernel


class _AdaLNNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, shift, scale, idx, eps):
        from vdn_minimax_h3_b200.ops import norm as norm_ops
        D = x.shape[1]
        table = torch.cat([shift, scale], dim=1).to(torch.bfloat16).contiguous()
        idx32 = idx.to(torch.int32).contiguous()
        w = None if weight is None else weight.detach().float().contiguous()
        out = norm_ops.adaln_rmsnorm(x, w, eps, table, 0, D, idx32)
        ctx.save_for_backward(x, table, idx32, w)
        ctx.eps = eps
        ctx.weight_dtype = None if weight is None else weight.dtype
        ctx.mod_dtypes = (shift.dtype, scale.dtype)
        return out

    @staticmethod
    def backward(ctx, dy):
        from vdn_minimax_h3_b200.ops._ext import ext
        x, table, idx32, w = ctx.saved_tensors
        D = x.shape[1]
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(x)
        ext().adaln_rmsnorm_bwd(x, dy, w, float(ctx.eps), table, D, idx32, dx)
        d_w = d_shift = d_scale = None
        need_w, need_shift, need_scale = ctx.needs_input_grad[1:4]
        if need_w or need_shift or need_scale:
            xf, dyf = x.float(), dy.float()
            xh = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + ctx.eps)
            idx = idx32.long()
            n = table.shape[0]
            if need_w:
                d_w = (dyf * xh * (1.0 + table[:, D:].float()[idx])).sum(0).to(ctx.weight_dtype)
            if need_shift:
                d_shift = torch.zeros(n, D, device=x.device).index_add_(0, idx, dyf)
                d_shift = d_shift.to(ctx.mod_dtypes[0])
            if need_scale:
                wf = 1.0 if w is None else w
                d_scale = torch.zeros(n, D, device=x.device).index_add_(0, idx, dyf * xh * wf)
                d_scale = d_scale.to(ctx.mod_dtypes[1])
        return dx, d_w, d_shift, d_scale, None, None


def adaln_modulated_norm(norm, x, shift, scale, idx):
    """norm(x) * (1 + scale[idx]) + shift[idx] for `norm` an RMSNorm module (weight, eps);
    x [..., T, D], shift / scale [n, D], idx [T]."""
    D = x.shape[-1]
    x2 = x.reshape(-1, D)
    if (NORM_KERNELS and x.is_cuda and x.dtype == torch.bfloat16
            and shift.dtype == torch.bfloat16 and scale.dtype == torch.bfloat16
            and D % 8 == 0 and D <= MAX_DIM and x2.shape[0] == idx.numel()
            and x2.stride(1) == 1 and (x2.stride(0) * 2) % 16 == 0 and x2.data_ptr() % 16 == 0):
        return _AdaLNNorm.apply(x2, norm.weight, shift, scale, idx, float(norm.eps)).view(x.shape)
    return norm(x) * (1.0 + scale.index_select(0, idx)) + shift.index_select(0, idx)
