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


def matmul_layout(a, b, a_mn=False, b_mn=False, out=None, accumulate=False):
    """out (+)= op(a) @ op(b)^T on the tcgen05 GEMM, where op(a) = a.T when `a_mn` (a held as
    [K, M]) and op(b)^T = b when `b_mn` (b held as [K, N]); otherwise a is [M, K] and b is
    [N, K] as in `linear`. No transposed copy is made: the kernel reads the MN-major operand
    in its stored layout. CPU tensors take the fp32 oracle."""
    am = a.t() if a_mn else a
    bm = b if b_mn else b.t()
    M, N = am.shape[0], bm.shape[1]
    if not a.is_cuda:
        y = am.float() @ bm.float()
        if out is None:
            return y.to(a.dtype)
        out.copy_(((out.float() + y) if accumulate else y).to(out.dtype))
        return out
    if out is None:
        assert not accumulate
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    ext().gemm_bf16_layout(a, b, out, bool(a_mn), bool(b_mn), bool(accumulate), error_word(a.device))
    return out


def linear_dgrad(dy, weight, out=None):
    """Input gradient of y = x W^T: dx = dy @ W, with W [out, in] read as the MN-major
    [K=out, N=in] operand."""
    return matmul_layout(dy, weight, a_mn=False, b_mn=True, out=out)


def linear_wgrad(dy, x, out=None, accumulate=False):
    """Weight gradient of y = x W^T: dW = dy^T @ x [out, in], contracting over the rows (T):
    dy read as the MN-major [K=T, M=out] operand, x as [K=T, N=in]."""
    return matmul_layout(dy, x, a_mn=True, b_mn=True, out=out, accumulate=accumulate)


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


class ColumnRoute:
    """Where each 8-column group of a routed GEMM's output goes.

    The route has `planes` destination tables. `place(col, view, plane)` sends output
    columns [col, col + view.shape[1]) of every row r to view[r]; a column group placed in
    several planes is stored to each (a field replicated to several ranks). For the q/k
    head columns of `linear_routed`, plane 0 receives the raw projection and plane 1 the
    per-head RMSNorm + RoPE'd values. Views may live anywhere the GPU can store to: a local
    buffer, a slab of a Ulysses exchange buffer, or a peer GPU's buffer mapped into this
    process. The views of one plane share a row stride. Columns never placed are computed
    and dropped."""

    MAX_PLANES = 8

    def __init__(self, n_cols, planes=2):
        if n_cols % 8:
            raise ValueError("routed GEMM output width must be a multiple of 8")
        if not 1 <= planes <= self.MAX_PLANES:
            raise ValueError(f"1..{self.MAX_PLANES} planes")
        self.n_cols = n_cols
        self.entries = [[] for _ in range(planes)]
        self._dev = None

    @property
    def raw(self):
        return self.entries[0]

    @property
    def proc(self):
        return self.entries[1] if len(self.entries) > 1 else []

    def place(self, col, view, plane=0):
        w = view.shape[1]
        if col % 8 or w % 8 or col + w > self.n_cols:
            raise ValueError(f"columns [{col}, {col + w}) are not whole 8-column groups of "
                             f"[0, {self.n_cols})")
        if view.dim() != 2 or view.stride(1) != 1:
            raise ValueError("route destinations are 2-D views with contiguous rows")
        if view.is_cuda and view.dtype != torch.bfloat16:
            raise ValueError("CUDA route destinations are bf16")
        self.entries[plane].append((col, view))
        self._dev = None
        return self

    def tables(self, device):
        """(route [planes, N/8] int64 addresses on `device`, [row stride per plane])."""
        if self._dev is None:
            rows, lds = [], []
            for plane, entries in enumerate(self.entries):
                t = [0] * (self.n_cols // 8)
                ld = {v.stride(0) for _, v in entries}
                if len(ld) > 1:
                    raise ValueError(f"plane {plane} destinations need one row stride, "
                                     f"got {sorted(ld)}")
                for col, v in entries:
                    if v.data_ptr() % 16 or (v.stride(0) * 2) % 16:
                        raise ValueError("route destinations must be 16-byte aligned")
                    for g in range(v.shape[1] // 8):
                        t[col // 8 + g] = v.data_ptr() + 16 * g
                rows.append(t)
                lds.append(ld.pop() if ld else 8)
            self._dev = (torch.tensor(rows, dtype=torch.int64, device=device), lds)
        return self._dev

    def copy_from(self, y, processed=()):
        """Host-side semantics of the routed stores: every placed view receives its columns
        of y, except plane-1 views inside a `processed` range (col0, tensor), which receive
        the tensor's columns. Used on CPU and for head widths the fused epilogue lacks."""
        for plane, entries in enumerate(self.entries):
            for col, v in entries:
                src = y
                off = col
                if plane == 1:
                    for c0, t in processed:
                        if c0 <= col < c0 + t.shape[1]:
                            src, off = t, col - c0
                            break
                v.copy_(src[:, off:off + v.shape[1]])


def linear_routed(x, weight, bias, route, q_cols=(0, 0), k_cols=(0, 0), norm_q=None,
                  norm_k=None, qk_eps=1e-6, cos=None, sin=None):
    """y = x @ weight.T + bias, scattered through `route` (ColumnRoute). Columns in
    q_cols / k_cols are 128-wide heads: their raw values go to plane 0 and
    rms_norm(head) * norm_{q,k} followed by rotate-half RoPE (cos/sin [M, 128]) to plane 1.
    One GEMM replaces projection + QK-prep + the Ulysses pack."""
    qk = q_cols[1] > q_cols[0] or k_cols[1] > k_cols[0]
    if not x.is_cuda:
        from vdn_minimax_h3_b200.ops.norm import qk_prep_reference
        y = F.linear(x.float(), weight.float(), None if bias is None else bias.float())
        y = y.to(x.dtype)
        proc = []
        for (lo, hi), w in ((q_cols, norm_q), (k_cols, norm_k)):
            if hi > lo:
                proc.append((lo, qk_prep_reference(y[:, lo:hi], (hi - lo) // w.numel(), w,
                                                   qk_eps, cos, sin)))
        route.copy_from(y, proc)
        return route
    table, lds = route.tables(x.device)
    f32 = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    ext().gemm_bf16_routed(x, weight, _bias32(bias), table, lds, q_cols[0], q_cols[1],
                           k_cols[0], k_cols[1], f32(norm_q), f32(norm_k), float(qk_eps),
                           cos if qk else None, sin if qk else None, error_word(x.device))
    return route
