"""The bidirectional frame-wise delta-rule linear-attention branch and its small layers.

Reference parity (src/models/linear_attention/):
  RMSNorm (fp32 second moment)       ops/rms_norm.py:23-32
  OutputGate                         attention_gates.py:13-55
  FrameKDAAlpha                      layers.py:12-69
  LinearAttentionSepConv             features.py:133-209 (5x5 depthwise spatial, then a
                                     5-tap depthwise temporal conv, both bias-free)
  BidirectionalLinearBranch          branch.py:46-458 (text state 0.5*S_text, skip_ends,
                                     head-sliced inference body for Ulysses)

Parameter names and shapes are the reference's, so v2 checkpoints load unchanged.

Two bodies, chosen by the caller (`inference=`), never by ambient grad state:
  _readout            eager PyTorch, differentiable: the training body and the oracle. Its
                      SPD factor and scans go through ops/linear_branch_grad.py (sm_100a
                      kernels forward and an adjoint-scan backward on CUDA with d = 128;
                      linear_branch_grad.USE_KERNELS = False keeps them on PyTorch).
  _readout_inference  forward-only: on CUDA every stage is an sm_100a kernel
                      (ops/linear_branch.py); on CPU the same stages run their oracles.
"""
import math

import torch
import torch.nn.functional as F
from torch import nn

from vdn_minimax_h3_b200.models.delta_rule import DELTA_BACKENDS
from vdn_minimax_h3_b200.models.scan import (BRIDGE_MODES, frame_statistics,
                                             gather_linear_state)
from vdn_minimax_h3_b200.ops.linear_branch_grad import conv_features as conv_features_grad
from vdn_minimax_h3_b200.ops.linear_branch_grad import conv_kernel_ok, scans, vdn_factor

SHORT_CONV_TARGETS = ("q", "k", "v")


class RMSNorm(nn.Module):
    """nn.RMSNorm-compatible (weight [dim], ones-init) with an fp32 second moment."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        ms = torch.linalg.vector_norm(x, dim=-1, keepdim=True, dtype=torch.float32).pow(2) / x.shape[-1]
        return x * torch.rsqrt(ms + self.eps).to(x.dtype) * self.weight.to(x.dtype)


class OutputGate(nn.Module):
    """Sigmoid gate: per head (softmax side, constant init 0.99) or per channel low rank
    (linear side, live random init)."""

    def __init__(self, hidden_size, num_heads, head_dim=None, bottleneck=None,
                 init_value=0.9, init="constant"):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        out_features = num_heads * (head_dim or 1)
        self.down = None if bottleneck is None else nn.Linear(hidden_size, bottleneck, bias=False)
        self.up = nn.Linear(bottleneck or hidden_size, out_features, bias=True)
        if init == "constant":
            nn.init.zeros_(self.up.weight)
            nn.init.constant_(self.up.bias, math.log(init_value / (1.0 - init_value)))
        elif init != "random":
            raise ValueError(f"OutputGate init must be 'constant' or 'random', got {init!r}")

    def forward(self, x):
        gate = torch.sigmoid(self.up(x if self.down is None else self.down(x)))
        return gate.view(-1, self.num_heads, self.head_dim or 1)


class FrameKDAAlpha(nn.Module):
    """alpha = exp(-exp(A_log) * softplus(up(down(frame_mean)) + dt_bias)), fp32 island."""

    def __init__(self, hidden_size, num_heads, head_dim, bottleneck=None):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        bottleneck = bottleneck or head_dim
        self.down = nn.Linear(hidden_size, bottleneck, bias=False)
        self.up = nn.Linear(bottleneck, num_heads * head_dim, bias=False)
        self.A_log = nn.Parameter(torch.log(torch.empty(num_heads).uniform_(1, 16)))
        dt = torch.exp(torch.rand(num_heads * head_dim) * (math.log(0.1) - math.log(0.001))
                       + math.log(0.001)).clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))

    def forward(self, frame_mean_x, heads=None):
        if heads is None:
            up_w, dt_bias, a_log, n = self.up.weight, self.dt_bias, self.A_log, self.num_heads
        else:
            rows = slice(heads.start * self.head_dim, heads.stop * self.head_dim)
            up_w, dt_bias, a_log = self.up.weight[rows], self.dt_bias[rows], self.A_log[heads]
            n = heads.stop - heads.start
        with torch.autocast(device_type=frame_mean_x.device.type, enabled=False):
            delta = F.linear(frame_mean_x.float(), self.down.weight.float())
            delta = F.linear(delta, up_w.float()) + dt_bias.float()
            scale = torch.exp(a_log.float())[:, None]
            delta = delta.view(-1, n, self.head_dim)
            return torch.exp(-scale * F.softplus(delta.float()))


class LinearAttentionSepConv(nn.Module):
    """Depthwise 5x5 spatial then 5-tap temporal conv on the listed projections."""

    KERNEL = 5

    def __init__(self, channels, projs=("k", "v")):
        super().__init__()
        self.projs = tuple(projs)
        k = self.KERNEL
        for name in self.projs:
            sp = nn.Conv2d(channels, channels, k, padding=k // 2, groups=channels, bias=False)
            nn.init.normal_(sp.weight, std=(k * k) ** -0.5)
            tm = nn.Conv1d(channels, channels, k, padding=k // 2, groups=channels, bias=False)
            nn.init.normal_(tm.weight, std=k ** -0.5)
            setattr(self, f"{name}_sp", sp)
            setattr(self, f"{name}_tm", tm)

    def weights(self, proj, channels=None):
        """(spatial [C, 5, 5], temporal [C, 5]) for one projection, optionally a channel slice."""
        sp = getattr(self, f"{proj}_sp").weight[:, 0]
        tm = getattr(self, f"{proj}_tm").weight[:, 0]
        if channels is not None:
            sp, tm = sp[channels], tm[channels]
        return sp, tm


def conv_features_reference(tokens, w_sp, w_tm, num_frames, frame_size, l2norm):
    """[F*S, H, d] -> separable conv -> SiLU [-> L2 over d]. Eager oracle, differentiable."""
    heads, head_dim = tokens.shape[-2:]
    gh, gw = frame_size
    C = heads * head_dim
    vol = tokens.reshape(num_frames, gh, gw, C).permute(0, 3, 1, 2)
    vol = F.conv2d(vol, w_sp.unsqueeze(1).to(vol.dtype), padding=2, groups=C)
    x = vol.permute(0, 2, 3, 1).reshape(num_frames, gh * gw, C)
    w = w_tm.to(x.dtype)
    xp = F.pad(x, (0, 0, 0, 0, 2, 2))
    out = None
    for dt in range(5):
        part = xp[dt:dt + num_frames] * w[:, dt].view(1, 1, -1)
        out = part if out is None else out + part
    return activate(out.reshape(-1, heads, head_dim), l2norm)


def activate(tokens, l2norm):
    x = F.silu(tokens)
    return F.normalize(x, dim=-1, eps=1e-6).to(x.dtype) if l2norm else x


class BidirectionalLinearBranch(nn.Module):
    TEXT_STATE_SCALE = 0.5

    def __init__(self, hidden_size, num_heads, head_dim, delta_rule="sana_scaled",
                 gate_bottleneck=None, bridge="alpha", a_fp32=True, short_conv=()):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        if bridge not in BRIDGE_MODES:
            raise ValueError(f"bridge {bridge!r} not in {BRIDGE_MODES}")
        self.bridge = bridge
        self.a_fp32 = a_fp32
        targets = tuple(short_conv) if isinstance(short_conv, (list, tuple)) else None
        if (targets is None or any(t not in SHORT_CONV_TARGETS for t in targets)
                or len(set(targets)) != len(targets)):
            raise ValueError(f"short_conv={short_conv!r}; expected a distinct subset of "
                             f"{SHORT_CONV_TARGETS}")
        self.short_conv = LinearAttentionSepConv(num_heads * head_dim, targets) if targets else None
        self.alpha = FrameKDAAlpha(hidden_size, num_heads, head_dim)
        self.beta_proj = nn.Linear(hidden_size, num_heads, bias=False)
        self.output_gate = OutputGate(hidden_size, num_heads, head_dim,
                                      bottleneck=gate_bottleneck or head_dim, init="random")
        self.norm = RMSNorm(head_dim)
        if delta_rule not in DELTA_BACKENDS:
            raise ValueError(f"delta_rule {delta_rule!r} not in {tuple(DELTA_BACKENDS)}")
        self.delta_rule = delta_rule
        self.checkpoint_features = False

    # ------------------------------------------------------------------ shared pieces
    def backend(self, length):
        return DELTA_BACKENDS[self.delta_rule](length)

    def feature(self, tokens, proj, num_frames, frame_size, use_conv=True, channels=None):
        conv = self.short_conv if use_conv else None
        l2 = proj != "v"
        if conv is not None and proj in conv.projs:
            if frame_size is None:
                raise ValueError("short_conv needs the spatial grid; pass frame_size=(H, W)")
            w_sp, w_tm = conv.weights(proj, channels)
            if conv_kernel_ok(tokens, frame_size):
                # sm_100a two-pass forward, conv_bwd.cu backward
                return conv_features_grad(tokens, w_sp, w_tm, num_frames, frame_size, l2)
            return conv_features_reference(tokens, w_sp, w_tm, num_frames, frame_size, l2)
        return activate(tokens, l2)

    def text_state(self, text_x, text_qkv_raw, heads=None, text_beta=None, channels=None):
        """TEXT_STATE_SCALE * S_text ([H, d, d] fp32), or None without a prompt."""
        if text_x is None and text_beta is None:
            return None
        n = self.num_heads if heads is None else heads.stop - heads.start
        d = self.head_dim
        L = text_qkv_raw[1].shape[0]
        key = activate(text_qkv_raw[1], True).view(1, L, n, d).permute(0, 2, 1, 3)
        value = activate(text_qkv_raw[2], False).view(1, L, n, d).permute(0, 2, 1, 3)
        beta = torch.sigmoid(self.beta_proj(text_x)) if text_beta is None else text_beta
        beta = beta.reshape(1, L, n).permute(0, 2, 1)
        A, B = frame_statistics(key, value, beta, a_fp32=self.a_fp32)
        with torch.autocast(device_type=A.device.type, enabled=False):
            ones = torch.ones(1, n, d, device=A.device, dtype=A.dtype)
            _, inj = self.backend(L).factor_apply(ones, A, B)
        return self.TEXT_STATE_SCALE * inj[0]

    # ------------------------------------------------------------------------ forward
    def forward(self, xv, num_frames, tokens_per_frame, bounds, qkv_raw, frame_size=None,
                skip_ends=False, text_x=None, text_qkv_raw=None, inference=False, heads=None,
                beta=None, gate=None, frame_mean=None, text_beta=None):
        """Linear readout [F*S, H*d] for every video row (the anchor frames read zero when
        `skip_ends`). See the reference's branch.py:218-324 for the contract."""
        if inference and torch.is_grad_enabled():
            raise RuntimeError("inference=True inside an enabled-grad region; wrap the forward "
                               "in torch.no_grad() or use the training body")
        sharded = dict(heads=heads, beta=beta, gate=gate, frame_mean=frame_mean,
                       text_beta=text_beta)
        if any(v is not None for v in sharded.values()) and not inference:
            raise ValueError("heads/beta/gate/frame_mean/text_beta are inference-only")
        run = ((lambda *a: self._readout_inference(*a, **sharded)) if inference
               else self._readout)
        n_heads = self.num_heads if heads is None else heads.stop - heads.start
        ref = xv if xv is not None else gate
        if not skip_ends:
            return run(xv, num_frames, tokens_per_frame, bounds, qkv_raw, frame_size,
                       text_x, text_qkv_raw)
        if num_frames <= 2:
            return ref.new_zeros(num_frames * tokens_per_frame, n_heads * self.head_dim)
        inner = slice(tokens_per_frame, (num_frames - 1) * tokens_per_frame)
        if inference:
            sharded.update(beta=None if beta is None else beta[inner],
                           gate=None if gate is None else gate[inner],
                           frame_mean=None if frame_mean is None else frame_mean[1:-1])
            run = lambda *a: self._readout_inference(*a, **sharded)  # noqa: E731
        readout = run(None if xv is None else xv[inner], num_frames - 2, tokens_per_frame,
                      [(lo - 1, hi - 1) for lo, hi in bounds[1:num_frames - 1]],
                      tuple(t[inner] for t in qkv_raw), frame_size, text_x, text_qkv_raw)
        out = readout.new_empty(num_frames * tokens_per_frame, readout.shape[-1])
        out[:tokens_per_frame].zero_()
        out[(num_frames - 1) * tokens_per_frame:].zero_()
        out[inner] = readout
        return out

    def _readout(self, xv, num_frames, tokens_per_frame, bounds, qkv_raw, frame_size=None,
                 text_x=None, text_qkv_raw=None):
        """The training body (eager, differentiable)."""
        F_, S, H, d = num_frames, tokens_per_frame, self.num_heads, self.head_dim
        shape = (F_, S, H, d)
        q, k, v = (self.feature(t, p, F_, frame_size) for t, p in zip(qkv_raw, "qkv"))
        qf = q.view(shape)
        kf = k.view(shape).permute(0, 2, 1, 3)
        vf = v.view(shape).permute(0, 2, 1, 3)
        beta = torch.sigmoid(self.beta_proj(xv)).view(F_, S, H).permute(0, 2, 1)
        A, B = frame_statistics(kf, vf, beta, a_fp32=self.a_fp32)
        alpha = self.alpha(xv.view(F_, S, -1).mean(dim=1, dtype=torch.float32))
        text_state = self.text_state(text_x, text_qkv_raw)
        with torch.autocast(device_type=A.device.type, enabled=False):
            # sm_100a SPD-factor and scan kernels forward, adjoint recurrence backward
            trans, inj = vdn_factor(self.backend(S), alpha, A, B)
            prefix, suffix = scans(trans, inj, text_state)
        state = gather_linear_state(prefix, suffix, alpha, bounds, bridge=self.bridge,
                                    text_state=text_state).to(xv.dtype)
        readout = torch.einsum("fhvk,fshk->fshv", state, qf)
        readout = self.norm(readout.reshape(F_ * S, H, d))
        return (readout * self.output_gate(xv)).reshape(F_ * S, H * d)

    def _readout_inference(self, xv, num_frames, tokens_per_frame, bounds, qkv_raw,
                           frame_size=None, text_x=None, text_qkv_raw=None, heads=None,
                           beta=None, gate=None, frame_mean=None, text_beta=None):
        """Forward-only body over a head range; every stage goes through ops.linear_branch
        (sm_100a kernels on CUDA)."""
        from vdn_minimax_h3_b200.ops import linear_branch as lb
        F_, S, d = num_frames, tokens_per_frame, self.head_dim
        n = self.num_heads if heads is None else heads.stop - heads.start
        channels = (slice(None) if heads is None
                    else slice(heads.start * d, heads.stop * d))
        conv = self.short_conv
        feats = []
        for t, proj in zip(qkv_raw, "qkv"):
            if conv is not None and proj in conv.projs:
                w_sp, w_tm = conv.weights(proj, channels)
                feats.append(lb.conv_features(t, w_sp, w_tm, F_, frame_size, proj != "v"))
            else:
                feats.append(lb.activate(t, proj != "v"))
        q, k, v = feats
        if beta is None:
            beta = torch.sigmoid(F.linear(xv, self.beta_proj.weight))
        A, B = lb.frame_statistics(k.view(F_, S, n, d), v.view(F_, S, n, d),
                                   beta.reshape(F_, S, n), a_fp32=self.a_fp32)
        del k, v
        if frame_mean is None:
            frame_mean = xv.view(F_, S, -1).mean(dim=1, dtype=torch.float32)
        alpha = self.alpha(frame_mean, heads=heads)
        text_state = self.text_state(text_x, text_qkv_raw, heads=heads, text_beta=text_beta,
                                     channels=channels)
        trans, inj = lb.factor_apply(self.backend(S), alpha, A, B)
        prefix, suffix = lb.run_scans(trans, inj, text_state)
        if gate is None:
            gate = self.output_gate(xv)
        state = lb.gather(prefix, suffix, alpha, bounds, self.bridge, text_state,
                          out_dtype=q.dtype)
        del prefix, suffix
        return lb.readout(q.view(F_, S, n, d), state, self.norm.weight, gate.reshape(F_ * S, n, d),
                          self.norm.eps)
