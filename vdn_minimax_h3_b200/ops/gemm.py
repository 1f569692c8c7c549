"""Linear layers on the tcgen05 GEMM (csrc/gemm.cu), with the fused epilogues of the DiT
block. CPU tensors take the fp32 PyTorch oracle (the numerics the kernels are tested
against); CUDA tensors always run the kernel.

Reference parity: the epilogues replace the pointwise stretches of
src/models/ops/fused_block.py:41-90 (gated residual, SwiGLU) and the plain nn.Linear /
cuBLAS calls of the block (L3/L4 in the reference's kernel inventory).
"""
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops._ext import error_word, ext


def _bias32(bias):
    if bias is None:
        return None
    return bias if bias.dtype == torch.float32 and bias.is_contiguous() else bias.float().contiguous()


def linear(x, weight, bias=None, out=None, accumulate=False):
    """out (+)= x @ weight.T (+ bias). x [M, K], weight [N, K] (bf16 on CUDA)."""
    if not x.is_cuda:
        y = F.linear(x.float(), weight.float(), None if bias is None else bias.float())
        if out is None:
            return y.to(x.dtype)
        if accumulate:
            out.copy_((out.float() + y).to(out.dtype))
        else:
            out.copy_(y.to(out.dtype))
        return out
    if out is None:
        assert not accumulate
        out = torch.empty(x.shape[0], weight.shape[0], dtype=torch.bfloat16, device=x.device)
    ext().gemm_bf16(x, weight, out, _bias32(bias), accumulate, error_word(x.device))
    return out


def linear_gated_residual(x, weight, bias, residual, gate_table, gate_index):
    """residual += gate_table[gate_index] * (x @ weight.T + bias), in place; returns residual.
    The fused `post` of the block (reference fused_block.py:47-49)."""
    if not x.is_cuda:
        y = F.linear(x.float(), weight.float(), None if bias is None else bias.float())
        g = gate_table.float().index_select(0, gate_index.long())
        residual.copy_((residual.float() + g * y).to(residual.dtype))
        return residual
    ext().gemm_bf16_residual(x, weight, residual, _bias32(bias), gate_table,
                             gate_index, error_word(x.device))
    return residual


def interleave_swiglu_rows(weight, bias=None, tile=256):
    """[2I, K] projection packed [value; gate] (diffusers' SwiGLU order) -> the kernel's
    layout: per `tile` rows, tile/2 value rows then the matching tile/2 gate rows."""
    two_i = weight.shape[0]
    inter = two_i // 2
    half = tile // 2
    assert inter % half == 0, f"intermediate {inter} not a multiple of {half}"
    v = weight[:inter].reshape(inter // half, half, -1)
    g = weight[inter:].reshape(inter // half, half, -1)
    w = torch.stack([v, g], dim=1).reshape(two_i, -1).contiguous()
    if bias is None:
        return w, None
    bv = bias[:inter].reshape(inter // half, half)
    bg = bias[inter:].reshape(inter // half, half)
    return w, torch.stack([bv, bg], dim=1).reshape(two_i).contiguous()


def linear_swiglu(x, weight_interleaved, bias_interleaved=None, tile=256):
    """silu-gated FF projection: a * silu(g) where [a | g] = x @ W.T + b, with W given in
    `interleave_swiglu_rows` layout. Returns [M, I]."""
    n = weight_interleaved.shape[0]
    if not x.is_cuda:
        h = F.linear(x.float(), weight_interleaved.float(),
                     None if bias_interleaved is None else bias_interleaved.float())
        h = h.view(x.shape[0], n // tile, 2, tile // 2)
        out = h[:, :, 0] * F.silu(h[:, :, 1])
        return out.reshape(x.shape[0], n // 2).to(x.dtype)
    out = torch.empty(x.shape[0], n // 2, dtype=torch.bfloat16, device=x.device)
    ext().gemm_bf16_swiglu(x, weight_interleaved, out, _bias32(bias_interleaved),
                           error_word(x.device))
    return out
