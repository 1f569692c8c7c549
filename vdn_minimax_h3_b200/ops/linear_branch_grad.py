"""Differentiable stages of the linear branch for the training body.

The reference trains through autograd of its eager ops (src/models/linear_attention/scan.py:
170-255, delta_rule.py:31-89): the two serial recurrences are 2F dependent `baddbmm`
launches per layer forward, and autograd replays them backwards as another ~4F launches
plus a Cholesky backward per frame. Here both stages are `torch.autograd.Function`s:

* `scans(trans, inj, start)`: forward runs the sm_100a scan kernel (both recurrences in
  one launch). The backward is the adjoint recurrence, which has the same shape as the
  forward one. With P_t = P_{t-1} T_t + J_t (prefix, t = 0..F-1, P_{-1} = S0) and
  Q_t = Q_{t+1} T_t + J_t (suffix, Q_F = S0), and upstream gradients gP, gQ:

      G_t = gP_t + G_{t+1} T_{t+1}^T     (G_F = 0, runs backwards in time)
      K_t = gQ_t + K_{t-1} T_{t-1}^T     (K_{-1} = 0, runs forwards)
      dJ_t = G_t + K_t
      dT_t = P_{t-1}^T G_t + Q_{t+1}^T K_t
      dS0  = G_0 T_0^T + K_{F-1} T_{F-1}^T

  G is run time-reversed, so both adjoints are prefix recurrences; they are stacked as 2H
  heads and the scan kernel runs them in one prefix-only launch. dT is a batched product
  (parallel over frames, off the serial path).
* `vdn_factor(backend, alpha, A, B)`: forward X = (I + a sym(A))^-1 and inj = b B X from the
  SPD kernel (Gauss-Jordan), T = diag(alpha) X. Backward from the saved X:

      dX = diag(alpha) dT + b B^T dinj,  dalpha = rowsum(dT * X),  dB = b dinj X,
      dA = -a sym(X dX X)               (X symmetric)

* `conv_features(tokens, w_sp, w_tm, F, frame_size, l2)`: the short conv's forward runs the
  two-pass kernels (5x5 spatial into a bf16 intermediate, then 5-tap temporal + SiLU [+ L2]),
  keeping the intermediate; the backward runs conv_bwd.cu (temporal + activation backward
  with the temporal weight gradient, then the flipped 5x5 stencil with the spatial weight
  gradient). Needs bf16 [N, H, 128] rows and a grid row of at most 44 positions; anything
  else, and CPU tensors, runs the eager PyTorch conv through autograd.

On CPU tensors, or a head dim other than 128, the same Functions run the fp32 PyTorch
recurrences (no kernel), so the adjoint formulas are tested against autograd on CPU.
"""
import torch

from vdn_minimax_h3_b200.models.scan import run_scans
from vdn_minimax_h3_b200.models.delta_rule import VdnDelta


# False: the CUDA path runs the PyTorch recurrences too (the oracle for kernel tests).
USE_KERNELS = True


def _kernel_path(t):
    return USE_KERNELS and t.is_cuda and t.shape[-1] == 128 and t.shape[-2] == 128


def _f32(t):
    """fp32, or fp64 kept as is (the gradient checks run in double)."""
    return t if t.dtype == torch.float64 else t.float()


def _prefix_scan(trans, inj):
    """P_t = P_{t-1} T_t + J_t from P_{-1} = 0, [F, n, d, d] fp32 (one direction)."""
    if _kernel_path(trans):
        from vdn_minimax_h3_b200.ops._ext import error_word, ext
        out = torch.empty_like(inj)
        ext().lb_scan(trans.contiguous(), inj.contiguous(), None, out, None,
                      error_word(trans.device))
        return out
    out = torch.empty_like(inj)
    state = torch.zeros_like(inj[0])
    for f in range(trans.shape[0]):
        state = torch.baddbmm(inj[f], state, trans[f])
        out[f] = state
    return out


def _forward_scans(trans, inj, start):
    if _kernel_path(trans):
        from vdn_minimax_h3_b200.ops import linear_branch as lb
        return lb.run_scans(trans, inj, start)
    return run_scans(trans, inj, start)


def scan_adjoint(trans, prefix, suffix, start, g_prefix, g_suffix):
    """(dJ, dT, dS0) of the two recurrences; see the module docstring."""
    F_, n = trans.shape[:2]
    Tt = trans.transpose(-1, -2)
    adj_t = torch.empty(F_, 2 * n, *trans.shape[2:], dtype=trans.dtype, device=trans.device)
    adj_t[0].zero_()                                   # multiplies the zero initial state
    if F_ > 1:
        adj_t[1:, :n] = Tt.flip(0)[:-1]                # reversed G: U_s = T_{F-s}^T
        adj_t[1:, n:] = Tt[:-1]                        # K: W_t = T_{t-1}^T
    adj_j = torch.empty_like(adj_t)
    adj_j[:, :n] = g_prefix.flip(0)
    adj_j[:, n:] = g_suffix
    out = _prefix_scan(adj_t, adj_j)
    G = out[:, :n].flip(0)
    K = out[:, n:]
    d_inj = G + K
    d = trans.shape[-1]

    def bmm(a, b):
        return torch.bmm(a.reshape(-1, d, d), b.reshape(-1, d, d)).view(a.shape)

    d_trans = torch.zeros_like(trans)
    if F_ > 1:
        d_trans[1:] = bmm(prefix[:-1].transpose(-1, -2), G[1:])
        d_trans[:-1] += bmm(suffix[1:].transpose(-1, -2), K[:-1])
    d_start = None
    if start is not None:
        st = start.to(trans.dtype).transpose(-1, -2)
        d_trans[0] += torch.matmul(st, G[0])
        d_trans[-1] += torch.matmul(st, K[-1])
        d_start = torch.matmul(G[0], Tt[0]) + torch.matmul(K[-1], Tt[-1])
    return d_inj, d_trans, d_start


class _Scans(torch.autograd.Function):
    @staticmethod
    def forward(ctx, trans, inj, start):
        with torch.no_grad():
            prefix, suffix = _forward_scans(trans, inj, start)
        ctx.save_for_backward(trans, prefix, suffix, start)
        ctx.has_start = start is not None
        return prefix, suffix

    @staticmethod
    def backward(ctx, g_prefix, g_suffix):
        trans, prefix, suffix, start = ctx.saved_tensors
        if g_prefix is None:
            g_prefix = torch.zeros_like(prefix)
        if g_suffix is None:
            g_suffix = torch.zeros_like(suffix)
        d_inj, d_trans, d_start = scan_adjoint(trans, prefix, suffix,
                                               start if ctx.has_start else None,
                                               g_prefix.to(prefix.dtype).contiguous(),
                                               g_suffix.to(prefix.dtype).contiguous())
        if ctx.has_start and d_start is not None:
            d_start = d_start.to(start.dtype)
        return d_trans, d_inj, (d_start if ctx.has_start else None)


def scans(trans, inj, start=None):
    """Differentiable prefix / suffix banks, [F, n, d, d] fp32 (see the module docstring)."""
    if start is not None:
        start = _f32(start)
    return _Scans.apply(_f32(trans).contiguous(), _f32(inj).contiguous(), start)


def _factor_forward(alpha, A, B, a_scale, b_scale):
    if _kernel_path(A):
        from vdn_minimax_h3_b200.ops._ext import error_word, ext
        X = torch.empty_like(A)
        inj = torch.empty_like(A)
        ones = torch.ones(alpha.shape, dtype=torch.float32, device=A.device)
        ext().lb_spd_factor(A.contiguous(), B.contiguous(), ones, X, inj,
                            float(a_scale), float(b_scale), error_word(A.device))
        return X, inj
    eye = torch.eye(A.shape[-1], dtype=A.dtype, device=A.device)
    M = eye + a_scale * 0.5 * (A + A.transpose(-1, -2))
    chol = torch.linalg.cholesky(M)
    X = torch.cholesky_inverse(chol)
    return X, (b_scale * B) @ X


class _VdnFactor(torch.autograd.Function):
    @staticmethod
    def forward(ctx, alpha, A, B, a_scale, b_scale):
        with torch.no_grad():
            X, inj = _factor_forward(alpha, A, B, a_scale, b_scale)
            trans = alpha.unsqueeze(-1) * X
        ctx.save_for_backward(alpha, B, X)
        ctx.scales = (a_scale, b_scale)
        return trans, inj

    @staticmethod
    def backward(ctx, d_trans, d_inj):
        alpha, B, X = ctx.saved_tensors
        a_scale, b_scale = ctx.scales
        dX = torch.zeros_like(X)
        d_alpha = d_B = None
        if d_trans is not None:
            d_trans = d_trans.to(X.dtype)
            dX += alpha.unsqueeze(-1) * d_trans
            d_alpha = (d_trans * X).sum(-1)
        if d_inj is not None:
            d_inj = d_inj.to(X.dtype)
            dX += b_scale * torch.matmul(B.transpose(-1, -2), d_inj)
            d_B = b_scale * torch.matmul(d_inj, X)
        dM = -torch.matmul(torch.matmul(X, dX), X)
        d_A = (0.5 * a_scale) * (dM + dM.transpose(-1, -2))
        return d_alpha, d_A, d_B, None, None


def vdn_factor(backend, alpha, A, B):
    """Differentiable (transition, injection) of the vdn rules; the sana rule is
    elementwise and stays on autograd."""
    if not isinstance(backend, VdnDelta):
        return backend.factor_apply(alpha, A, B)
    return _VdnFactor.apply(_f32(alpha), _f32(A).contiguous(), _f32(B).contiguous(),
                            float(backend.a_scale), float(backend.b_scale))


# ------------------------------------------------------------------------- short conv
CONV_MAX_ROW = 44        # widest grid row of the two-pass forward kernels


def conv_kernel_ok(tokens, frame_size):
    """Whether the short conv's training kernels take these rows."""
    return (USE_KERNELS and tokens.is_cuda and tokens.dtype == torch.bfloat16
            and tokens.dim() == 3 and tokens.shape[-1] == 128 and tokens.stride(2) == 1
            and tokens.stride(1) == 128 and (tokens.stride(0) * 2) % 16 == 0
            and tokens.data_ptr() % 16 == 0 and frame_size[1] <= CONV_MAX_ROW)


class _ConvFeatures(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, w_sp, w_tm, num_frames, gh, gw, l2norm):
        from vdn_minimax_h3_b200.ops._ext import error_word, ext
        C = tokens.shape[1] * tokens.shape[2]
        wsp_t = w_sp.detach().float().reshape(C, 25).t().contiguous()     # taps [25, C]
        wtm = w_tm.detach().float().reshape(C, 5).contiguous()
        out = torch.empty(tokens.shape, dtype=torch.bfloat16, device=tokens.device)
        tmp = torch.empty(tokens.shape, dtype=torch.bfloat16, device=tokens.device)
        ext().lb_conv_features(tokens, wsp_t.reshape(-1), wtm.reshape(-1), out, num_frames, gh, gw,
                               bool(l2norm), error_word(tokens.device), tmp)
        ctx.save_for_backward(tokens, tmp, wsp_t, wtm)
        ctx.meta = (num_frames, gh, gw, bool(l2norm), w_sp.shape, w_sp.dtype, w_tm.shape,
                    w_tm.dtype)
        return out

    @staticmethod
    def backward(ctx, d_out):
        from vdn_minimax_h3_b200.ops._ext import ext
        tokens, tmp, wsp_t, wtm = ctx.saved_tensors
        num_frames, gh, gw, l2norm, sp_shape, sp_dtype, tm_shape, tm_dtype = ctx.meta
        C = tokens.shape[1] * tokens.shape[2]
        d_out = d_out.to(torch.bfloat16).contiguous()
        dtmp = torch.empty(tokens.shape[0], C, dtype=torch.float32, device=tokens.device)
        dx = torch.empty(tokens.shape, dtype=torch.bfloat16, device=tokens.device)
        dwsp = torch.zeros(25, C, dtype=torch.float32, device=tokens.device)
        dwtm = torch.zeros(C, 5, dtype=torch.float32, device=tokens.device)
        ext().lb_conv_features_bwd(tokens, tmp, d_out, wsp_t.reshape(-1), wtm.reshape(-1), dtmp, dx,
                                   dwsp.view(-1), dwtm.view(-1), num_frames, gh, gw, l2norm)
        del dtmp
        return (dx, dwsp.t().reshape(sp_shape).to(sp_dtype), dwtm.reshape(tm_shape).to(tm_dtype),
                None, None, None, None)


def conv_features(tokens, w_sp, w_tm, num_frames, frame_size, l2norm):
    """Differentiable short conv on the kernels; callers check `conv_kernel_ok` first.
    tokens [F*S, H, 128] bf16, w_sp [C, 5, 5], w_tm [C, 5] -> [F*S, H, 128] bf16."""
    gh, gw = frame_size
    return _ConvFeatures.apply(tokens, w_sp, w_tm, int(num_frames), int(gh), int(gw),
                               bool(l2norm))

