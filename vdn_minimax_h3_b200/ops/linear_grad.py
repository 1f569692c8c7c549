"""Training Linears on the tcgen05 GEMM: forward, input gradient and weight gradient.

The three products of an nn.Linear in a training step all run on csrc/gemm.cu, each with
the operand layouts the tensors already have (no transposed copies):

    forward  y  = x W^T     A = x [T, in] and B = W [out, in], both K-major
    dgrad    dx = dy W      A = dy [T, out] K-major, B = W read MN-major as [K=out, N=in]
    wgrad    dW = dy^T x    A = dy read MN-major as [K=T, M=out], B = x as [K=T, N=in]

and the bias gradient is an fp32 column sum. `route_training_linears(model)` gives every
nn.Linear of a model this forward (an instance-level override: parameter names, state-dict
keys and FSDP2 sharding are unchanged); a Linear whose tensors the kernel does not take
(fp32 weights such as the fp32 alpha island, a feature count that is not a multiple of 8,
CPU tensors) runs F.linear. The module switch `LINEAR_KERNELS = False` sends every routed
Linear back to F.linear (the labelled library baseline of the training bench).

Reference parity: the reference trains every projection as a stock nn.Linear on cuBLAS
(e.g. src/models/hybrid_attention.py:100, `to_out_linear`), sharded by
src/training/fsdp_stage.py:392-451; the math is the same product, rounded once to bf16 from
an fp32 accumulator as cuBLAS does.
"""
import types

import torch
import torch.nn as nn
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops import gemm

LINEAR_KERNELS = True
STATS = {"kernel": 0, "fallback": 0}


def _rows_ok(t):
    return (t.dim() == 2 and t.stride(-1) == 1 and (t.stride(0) * 2) % 16 == 0
            and t.data_ptr() % 16 == 0)


def kernel_path_ok(x2, weight):
    """True when the GEMM kernel takes y = x2 W^T and its two gradients."""
    return (LINEAR_KERNELS and x2.is_cuda and x2.dtype == torch.bfloat16
            and weight.dtype == torch.bfloat16 and weight.dim() == 2
            and x2.shape[-1] % 8 == 0 and weight.shape[0] % 8 == 0
            and _rows_ok(x2) and _rows_ok(weight))


def _bf16_rows(t):
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t if _rows_ok(t) else t.contiguous()


class _KernelLinear(torch.autograd.Function):
    """y = x2 W^T (+ b) with x2 [T, in]; backward dgrad / wgrad on the GEMM kernel."""

    @staticmethod
    def forward(ctx, x2, weight, bias):
        ctx.save_for_backward(x2, weight)
        ctx.bias_dtype = None if bias is None else bias.dtype
        return gemm.linear(x2, weight, bias)

    @staticmethod
    def backward(ctx, dy):
        x2, weight = ctx.saved_tensors
        dy = _bf16_rows(dy) if dy.is_cuda else dy
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = gemm.linear_dgrad(dy, weight)
        if ctx.needs_input_grad[1]:
            dw = gemm.linear_wgrad(dy, x2).to(weight.dtype)
        if ctx.bias_dtype is not None and ctx.needs_input_grad[2]:
            db = dy.float().sum(0).to(ctx.bias_dtype)
        return dx, dw, db


def kernel_linear(x, weight, bias=None):
    """F.linear(x, weight, bias) for x [..., in] on the GEMM kernel (forward and backward)
    when `kernel_path_ok`, else F.linear."""
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    if x2.is_cuda and x2.dtype == torch.bfloat16 and not _rows_ok(x2):
        x2 = x2.contiguous()
    if not kernel_path_ok(x2, weight):
        STATS["fallback"] += 1
        return F.linear(x, weight, bias)
    STATS["kernel"] += 1
    y = _KernelLinear.apply(x2, weight, bias)
    return y.view(*x.shape[:-1], weight.shape[0])


def _routed_forward(self, x):
    return kernel_linear(x, self.weight, self.bias)


def route_training_linears(model):
    """Every nn.Linear of `model` runs `kernel_linear` (forward + dgrad + wgrad on the GEMM
    kernel). Returns the number of Linears routed."""
    n = 0
    for m in model.modules():
        if type(m) is nn.Linear and getattr(m, "_vdn_kernel_linear", None) != "train":
            m.forward = types.MethodType(_routed_forward, m)
            m._vdn_kernel_linear = "train"
            n += 1
    return n
