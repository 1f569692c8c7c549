"""Block-scaled fp8 (E4M3) linears on the tcgen05 block-scaled MMA (csrc/gemm_fp8.cu).

Reference parity: src/models/ops/fp8_linear.py (Fp8Linear, the row / tensor quantisers and
the SwiGLU+quantise fusion). Here every scale is a power of two (UE8M0) so the tensor core
applies it during the MMA: activations get one scale per 1x128 block (quantised by the
kernel that produces them, or `quantize_act`), weights one per 128x128 block, quantised
once at load; the SwiGLU epilogue emits the next GEMM's E4M3 operand with one scale per
1x64 block. Scale factors are stored in the blocked layout the MMA's TMEM copies read:
128-row x 4-block atoms of 512 bytes, byte (r % 32) * 16 + (r % 128 // 32) * 4 + kb % 4
(csrc/common.cuh: sf_offset); weights are grouped per 256-row GEMM tile.

CPU tensors take the fp32 oracle (dequantise, matmul) these kernels are tested against.
"""
import torch
import torch.nn.functional as F

from vdn_minimax_h3_b200.ops._ext import error_word, ext

E4M3_MAX = 448.0
FP8 = torch.float8_e4m3fn


def e8_exponent(amax):
    """Smallest integer e with amax / 2^e <= 448, clamped to [-127, 127] (int32 tensor)."""
    v = amax.float() / E4M3_MAX
    m, k = torch.frexp(v)
    e = torch.where(m == 0.5, k - 1, k)
    e = torch.where(v < 2.0 ** -126, torch.full_like(e, -127), e)
    return e.clamp(-127, 127).to(torch.int32)


def _pow2(e):
    return torch.pow(2.0, e.float())


def quantize_blocks(x, block_rows, block_cols=128):
    """x [R, K] -> (E4M3 [R, K], exponents [ceil(R / block_rows), K / block_cols])."""
    R, K = x.shape
    assert K % block_cols == 0
    rb = (R + block_rows - 1) // block_rows
    xp = torch.zeros(rb * block_rows, K, dtype=torch.float32, device=x.device)
    xp[:R] = x.float()
    amax = xp.abs().view(rb, block_rows, K // block_cols, block_cols).amax(dim=(1, 3))
    e = e8_exponent(amax)
    inv = _pow2((-e).clamp(-126, 127))
    scale_rows = inv.repeat_interleave(block_rows, 0)[:R].repeat_interleave(block_cols, 1)
    q = (x.float() * scale_rows).to(FP8)
    return q, e


def _sf_index(rows, kb32, kb_total, tile_rows):
    """Byte offsets of (row, 32-block) scale factors; tile_rows = 128 (A) or 256 (B)."""
    r = rows[:, None]
    kb = kb32[None, :]
    per_tile = (tile_rows // 128) * 512
    return (((r // tile_rows) * (kb_total // 4) + kb // 4) * per_tile + ((r % tile_rows) // 128) * 512
            + (r % 32) * 16 + ((r % 128) // 32) * 4 + kb % 4)


def sf_blocked(e_rows, tile_rows):
    """Per-(row, 32-block) exponents [R, K/32] -> blocked UE8M0 bytes (rows padded)."""
    R, kb_total = e_rows.shape
    tiles = (R + tile_rows - 1) // tile_rows
    out = torch.full((tiles * (kb_total // 4) * (tile_rows // 128) * 512,), 127, dtype=torch.uint8,
                     device=e_rows.device)
    idx = _sf_index(torch.arange(R, device=e_rows.device), torch.arange(kb_total, device=e_rows.device),
                    kb_total, tile_rows)
    out[idx.reshape(-1)] = (e_rows + 127).to(torch.uint8).reshape(-1)
    return out


def sf_unblock(sf, R, K, tile_rows):
    """Inverse of sf_blocked: exponents [R, K/32] (int32)."""
    kb_total = K // 32
    idx = _sf_index(torch.arange(R, device=sf.device), torch.arange(kb_total, device=sf.device),
                    kb_total, tile_rows)
    return sf[idx.reshape(-1)].view(R, kb_total).to(torch.int32) - 127


def dequantize(q, sf, tile_rows):
    """E4M3 [R, K] + blocked scale factors -> fp32 [R, K]."""
    R, K = q.shape
    e = sf_unblock(sf, R, K, tile_rows)
    return q.view(FP8).float() * _pow2(e).repeat_interleave(32, 1)


class Fp8Weight:
    """A Linear weight quantised once: E4M3 [N, K] with one scale per 128x128 block."""

    def __init__(self, weight, bias=None, block=128):
        N, K = weight.shape
        if K % 128 or N % 32:
            raise ValueError(f"fp8 weights need K % 128 == 0 and N % 32 == 0, got {tuple(weight.shape)}")
        q, e = quantize_blocks(weight.detach(), block, 128)
        e_rows = e.repeat_interleave(block, 0)[:N].repeat_interleave(4, 1)
        self.q = q.view(torch.uint8).contiguous()
        self.sf = sf_blocked(e_rows, 256)
        self.bias = None if bias is None else bias.detach().float().contiguous()
        self.shape = (N, K)

    def dequantized(self):
        return dequantize(self.q, self.sf, 256)


def quantize_act(x, out=None, sf=None):
    """bf16 [M, K] -> (E4M3 [M, K] as uint8, blocked scale factors), one scale per 1x128."""
    M, K = x.shape
    if not x.is_cuda:
        q, e = quantize_blocks(x, 1, 128)
        return q.view(torch.uint8), sf_blocked(e.repeat_interleave(4, 1), 128)
    if out is None:
        out = torch.empty(M, K, dtype=torch.uint8, device=x.device)
    if sf is None:
        sf = torch.empty(((M + 127) // 128) * (K // 128) * 512, dtype=torch.uint8, device=x.device)
    ext().quant_rows(x, out, sf)
    return out, sf


def sf_bytes(M, K):
    return ((M + 127) // 128) * (K // 128) * 512


def _oracle(xq, xsf, w):
    a = dequantize(xq, xsf, 128)
    return a @ w.dequantized().t()


def linear_fp8(xq, xsf, w: Fp8Weight, out=None):
    """out = dequant(xq) @ dequant(w)^T + bias (bf16 [M, N])."""
    M, N = xq.shape[0], w.shape[0]
    if not xq.is_cuda:
        y = _oracle(xq, xsf, w)
        if w.bias is not None:
            y = y + w.bias
        y = y.to(torch.bfloat16)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=xq.device)
    ext().gemm_fp8(xq, w.q, xsf, w.sf, 0, out, w.bias, None, None, None, None, error_word(xq.device))
    return out


def linear_fp8_gated_residual(xq, xsf, w: Fp8Weight, residual, gate_table, gate_index):
    """residual += gate_table[gate_index] * (dequant(xq) @ dequant(w)^T + bias)."""
    if not xq.is_cuda:
        y = _oracle(xq, xsf, w)
        if w.bias is not None:
            y = y + w.bias
        g = gate_table.float().index_select(0, gate_index.long())[:, :y.shape[1]]
        residual.copy_((residual.float() + g * y).to(residual.dtype))
        return residual
    ext().gemm_fp8(xq, w.q, xsf, w.sf, 1, residual, w.bias, gate_table, gate_index, None, None,
                   error_word(xq.device))
    return residual


def linear_fp8_swiglu(xq, xsf, w: Fp8Weight, q_out=None, q_sf=None):
    """SwiGLU of an fp8 projection whose weight rows are interleaved per 128 as
    [64 value | 64 gate] (gemm.interleave_swiglu_rows(..., tile=128)); returns the E4M3
    output [M, N/2] and its blocked scale factors (one scale per 1x64 block)."""
    M, N = xq.shape[0], w.shape[0]
    if not xq.is_cuda:
        y = _oracle(xq, xsf, w)
        if w.bias is not None:
            y = y + w.bias
        y = y.view(M, N // 128, 2, 64)
        h = (y[:, :, 0] * F.silu(y[:, :, 1])).reshape(M, N // 2)
        q, e = quantize_blocks(h, 1, 64)
        return q.view(torch.uint8), sf_blocked(e.repeat_interleave(2, 1), 128)
    if q_out is None:
        q_out = torch.empty(M, N // 2, dtype=torch.uint8, device=xq.device)
    if q_sf is None:
        q_sf = torch.empty(sf_bytes(M, N // 2), dtype=torch.uint8, device=xq.device)
    ext().gemm_fp8(xq, w.q, xsf, w.sf, 2, None, w.bias, None, None, q_out, q_sf,
                   error_word(xq.device))
    return q_out, q_sf


def linear_routed_fp8(xq, xsf, w: Fp8Weight, route, q_cols=(0, 0), k_cols=(0, 0), norm_q=None,
                      norm_k=None, qk_eps=1e-6, cos=None, sin=None):
    """The routed projection (ops.gemm.linear_routed) on the block-scaled fp8 GEMM."""
    qk = q_cols[1] > q_cols[0] or k_cols[1] > k_cols[0]
    if not xq.is_cuda:
        from vdn_minimax_h3_b200.ops.norm import qk_prep_reference
        y = _oracle(xq, xsf, w)
        if w.bias is not None:
            y = y + w.bias
        y = y.to(torch.bfloat16)
        proc = []
        for (lo, hi), nw in ((q_cols, norm_q), (k_cols, norm_k)):
            if hi > lo:
                proc.append((lo, qk_prep_reference(y[:, lo:hi], (hi - lo) // nw.numel(), nw,
                                                   qk_eps, cos, sin)))
        route.copy_from(y, proc)
        return route
    table, lds = route.tables(xq.device)
    f32 = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    ext().gemm_fp8_routed(xq, w.q, xsf, w.sf, w.bias, table, lds, q_cols[0], q_cols[1],
                          k_cols[0], k_cols[1], f32(norm_q), f32(norm_k), float(qk_eps),
                          cos if qk else None, sin if qk else None, error_word(xq.device))
    return route


def trace_gemm_fp8(M=104766, N=21504, K=5376):  # pragma: no cover - GPU tool
    """Where the fp8 GEMM's MMA thread spends its cycles (per-CTA counters, averaged):
    waiting for staged operands, waiting for the accumulator to be drained, and the
    producer waiting for a free stage."""
    import json
    w8 = Fp8Weight(torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / 70)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    xq, xsf = quantize_act(x)
    out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    linear_fp8(xq, xsf, w8, out)
    tr = torch.zeros(4096, dtype=torch.int64, device="cuda")
    ext().gemm_fp8_set_trace(tr)
    try:
        linear_fp8(xq, xsf, w8, out)
        torch.cuda.synchronize()
    finally:
        ext().gemm_fp8_set_trace(None)
    t = tr.view(-1, 8)[:torch.cuda.get_device_properties(0).multi_processor_count].double()
    tot = t[:, 0].mean().item()
    res = {"mma_thread_cycles": tot, "wait_operands_frac": t[:, 1].mean().item() / tot,
           "wait_accumulator_frac": t[:, 2].mean().item() / tot,
           "producer_wait_stage_frac": t[:, 3].mean().item() / tot,
           "tiles_per_cta": t[:, 4].mean().item()}
    print(json.dumps({"gemm_fp8_trace": res}), flush=True)
    return res
