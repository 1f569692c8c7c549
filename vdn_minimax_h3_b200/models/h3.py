"""The MiniMax-H3 text-to-video+audio DiT backbone, re-implemented in PyTorch.

The reference never ships this model: it imports diffusers' MiniMaxH3Transformer3DModel
from a patched diffusers tree that is not part of it. What this file builds is pinned by
how the reference calls that model:
  * the forward is the one copied in src/inference/utils/ulysses.py:384-443 (embed, token
    refiner, packed index_copy, temb, per-row AdaLN index t_idx * MODALITY_NUM + tag,
    blocks, norm_out, the two output heads);
  * the block is the one in src/models/ops/fused_block.py:93-111 (RMSNorm + AdaLN affine,
    gated residual, SwiGLU feed-forward [value; gate]);
  * the AdaLN modulations run SiLU on temb in fp32 (diffusers_patches/0001-...patch:36-61);
  * the attention has to_q/to_k/to_v/to_out[0], per-head RMS QK-norm, then rotate-half
    RoPE on the first rotary_dim channels (softmax_attention/kernels.py:8-30).
Parameter NAMES follow the diffusers module tree those call sites use, so LoRA targets
(`transformer_blocks.N.attn.to_q`, `token_refiner.refiner_blocks.N.attn.to_q`, ...) and the
hybrid transform's `.attn.orig.` re-rooting resolve the same way.

Assumed where the reference is silent (fixed in H3Config):
time_embed_dim 3072 (this reproduces the ~33B parameter count), MODALITY_NUM 3, the rotary
split 32/48/48 channels over (t, h, w) with theta 10000, biases on every projection, a
two-block unconditioned self-attention token refiner, and LayerNorm-free RMS norm_out.
"""
import math
from dataclasses import asdict, dataclass, field
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from vdn_minimax_h3_b200.models.layout import MODALITY_NUM
from vdn_minimax_h3_b200.ops.norm_grad import adaln_modulated_norm


@dataclass
class H3Config:
    hidden_size: int = 5376
    num_layers: int = 50
    num_attention_heads: int = 56
    attention_head_dim: int = 128
    in_channels: int = 24
    patch_size: Tuple[int, int, int] = (1, 2, 2)
    audio_in_channels: int = 32
    text_dim: int = 5120
    time_embed_dim: int = 3072
    time_freq_dim: int = 256
    ff_inner_dim: int = 14336
    ff_activation: str = "swiglu"         # "swiglu" | "gelu"
    num_refiner_layers: int = 2
    rope_axes_dim: Tuple[int, int, int] = (32, 48, 48)
    rope_theta: float = 10000.0
    modality_num: int = MODALITY_NUM
    norm_eps: float = 1e-6
    qk_norm_eps: float = 1e-6

    @property
    def inner_dim(self):
        return self.num_attention_heads * self.attention_head_dim

    @property
    def rotary_dim(self):
        return sum(self.rope_axes_dim)

    def to_dict(self):
        d = asdict(self)
        d["patch_size"] = list(self.patch_size)
        d["rope_axes_dim"] = list(self.rope_axes_dim)
        return d

    @staticmethod
    def from_dict(d):
        d = {k: v for k, v in d.items() if k in H3Config.__dataclass_fields__}
        for k, f in H3Config.__dataclass_fields__.items():
            if k in d and f.type in (float, "float") and isinstance(d[k], str):
                d[k] = float(d[k])
        if "patch_size" in d:
            d["patch_size"] = tuple(d["patch_size"])
        if "rope_axes_dim" in d:
            d["rope_axes_dim"] = tuple(d["rope_axes_dim"])
        return H3Config(**d)


def h3_full_config():
    """The MiniMax-H3 geometry (50 blocks, 5376 wide, 56 x 128 heads)."""
    return H3Config()


def h3_tiny_config():
    """The tiny CPU configuration: 2 blocks, hidden 256, 4 heads of 64, GELU MLP 4x, 16 channels."""
    return H3Config(hidden_size=256, num_layers=2, num_attention_heads=4,
                    attention_head_dim=64, in_channels=16, audio_in_channels=32,
                    text_dim=256, time_embed_dim=256, time_freq_dim=64, ff_inner_dim=1024,
                    ff_activation="gelu", num_refiner_layers=1, rope_axes_dim=(16, 24, 24))


# ------------------------------------------------------------------------------ layers
class RMSNormAffine(nn.Module):
    def __init__(self, dim, eps=1e-6, affine=True):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim)) if affine else None

    def forward(self, x):
        w = None if self.weight is None else self.weight.to(x.dtype)
        return F.rms_norm(x, (x.shape[-1],), w, self.eps)


class Timesteps(nn.Module):
    """Sinusoidal embedding of t in [0, 1] (scaled to [0, 1000]), cos first."""

    def __init__(self, dim):
        super().__init__()
        self.dim = dim

    def forward(self, t):
        half = self.dim // 2
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device,
                                                            dtype=torch.float32) / half)
        args = (t.float() * 1000.0)[:, None] * freqs[None]
        return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


class TimestepEmbedding(nn.Module):
    def __init__(self, in_dim, dim):
        super().__init__()
        self.linear_1 = nn.Linear(in_dim, dim)
        self.linear_2 = nn.Linear(dim, dim)

    def forward(self, x):
        return self.linear_2(F.silu(self.linear_1(x)))


class RotaryEmbedding3D(nn.Module):
    """cos/sin [S, rotary_dim] from position_ids [S, 3]; rotate-half convention, each axis
    contributing axis_dim channels (half of them frequencies, duplicated)."""

    def __init__(self, axes_dim, theta=10000.0):
        super().__init__()
        self.axes_dim = tuple(axes_dim)
        self.theta = theta

    def forward(self, position_ids):
        freqs = []
        for axis, dim in enumerate(self.axes_dim):
            inv = 1.0 / (self.theta ** (torch.arange(0, dim, 2, device=position_ids.device,
                                                     dtype=torch.float32) / dim))
            freqs.append(position_ids[:, axis].float()[:, None] * inv[None])
        f = torch.cat(freqs, dim=-1)             # [S, rotary_dim / 2]
        f = torch.cat([f, f], dim=-1)            # rotate-half layout
        return torch.cos(f), torch.sin(f)


def apply_rotary_emb(x, cos, sin):
    """x [..., S, H, d]; rotate-half on the first cos.shape[-1] channels."""
    rot = cos.shape[-1]
    x_rot, x_pass = x[..., :rot], x[..., rot:]
    c = cos.to(x.dtype)[..., :, None, :]
    s = sin.to(x.dtype)[..., :, None, :]
    x1, x2 = x_rot.chunk(2, dim=-1)
    rotated = torch.cat((-x2, x1), dim=-1)
    return torch.cat((x_rot * c + rotated * s, x_pass), dim=-1)


class H3Attention(nn.Module):
    """to_q/to_k/to_v -> per-head RMS QK-norm -> RoPE -> dense softmax -> to_out."""

    def __init__(self, dim, heads, head_dim, eps=1e-6, bias=True):
        super().__init__()
        self.heads, self.head_dim = heads, head_dim
        inner = heads * head_dim
        self.to_q = nn.Linear(dim, inner, bias=bias)
        self.to_k = nn.Linear(dim, inner, bias=bias)
        self.to_v = nn.Linear(dim, inner, bias=bias)
        self.norm_q = RMSNormAffine(head_dim, eps)
        self.norm_k = RMSNormAffine(head_dim, eps)
        self.to_out = nn.ModuleList([nn.Linear(inner, dim, bias=bias), nn.Dropout(0.0)])

    def project(self, x, rotary_emb):
        """x [T, D] -> (q, k, v) [T, H, d] with QK-norm and RoPE, plus raw q, k."""
        q_raw = self.to_q(x).unflatten(-1, (self.heads, -1))
        k_raw = self.to_k(x).unflatten(-1, (self.heads, -1))
        v = self.to_v(x).unflatten(-1, (self.heads, -1))
        q, k = self.norm_q(q_raw), self.norm_k(k_raw)
        if rotary_emb is not None:
            q = apply_rotary_emb(q, *rotary_emb)
            k = apply_rotary_emb(k, *rotary_emb)
        return q, k, v, (q_raw, k_raw, v)

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        x = hidden_states[0]
        q, k, v, _ = self.project(x, rotary_emb)
        ag = _attention_kernels()
        if ag is not None and attention_mask is None and ag.kernel_path_ok(q, k, v):
            # dense attention (the teacher trunk, the refiner) on the sm_100a kernels
            o = ag.window_attention_train(q, k, v, ag.dense_plan(x.shape[0], x.device),
                                          q.shape[-1] ** -0.5).reshape(x.shape[0], -1)
        else:
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                               v.transpose(0, 1)[None], attn_mask=attention_mask)
            o = o[0].transpose(0, 1).reshape(x.shape[0], -1)
        return self.to_out[1](self.to_out[0](o)).unsqueeze(0)


def _attention_kernels():
    """ops.attention_grad when it is importable and switched on, else None (the exported
    single-file component, which carries no kernels, takes the SDPA path)."""
    try:
        from vdn_minimax_h3_b200.ops import attention_grad
    except ImportError:
        return None
    return attention_grad if attention_grad.ATTENTION_KERNELS else None


class SwiGLU(nn.Module):
    """a * silu(gate) with proj rows packed [value; gate]. After the inference engine packs
    the weight (`interleaved` = tile width), rows are interleaved per tile as
    [tile/2 value | tile/2 gate]; forward reads either layout."""

    def __init__(self, dim, inner, bias=True):
        super().__init__()
        self.proj = nn.Linear(dim, 2 * inner, bias=bias)
        self.interleaved = 0

    def forward(self, x):
        h = self.proj(x)
        if self.interleaved:
            t = self.interleaved
            h = h.unflatten(-1, (h.shape[-1] // t, 2, t // 2))
            return (h[..., 0, :] * F.silu(h[..., 1, :])).flatten(-2)
        a, gate = h.chunk(2, dim=-1)
        return a * F.silu(gate)


class GELUProj(nn.Module):
    def __init__(self, dim, inner, bias=True):
        super().__init__()
        self.proj = nn.Linear(dim, inner, bias=bias)

    def forward(self, x):
        return F.gelu(self.proj(x), approximate="tanh")


class FeedForward(nn.Module):
    """net = [activation projection, Dropout, down Linear] (diffusers' FeedForward)."""

    def __init__(self, dim, inner, activation="swiglu", bias=True):
        super().__init__()
        act = SwiGLU(dim, inner, bias) if activation == "swiglu" else GELUProj(dim, inner, bias)
        self.activation = activation
        self.net = nn.ModuleList([act, nn.Dropout(0.0), nn.Linear(inner, dim, bias=bias)])

    def forward(self, x):
        return self.net[2](self.net[1](self.net[0](x)))


class AdaLayerNormModulation(nn.Module):
    """Linear(temb -> 6 * hidden * MODALITY_NUM) on SiLU(temb) in fp32; rows are
    (timestep, modality), each 6 chunks (shift/scale/gate for attention, then for FF)."""

    def __init__(self, temb_dim, hidden, modality_num):
        super().__init__()
        self.hidden = hidden
        self.linear = nn.Linear(temb_dim, 6 * hidden * modality_num, bias=True)

    def table(self, temb):
        """[n_t, Dt] -> [n_t * MODALITY_NUM, 6 * hidden] in the projection's dtype."""
        w = self.linear.weight
        out = self.linear(F.silu(temb.float()).to(w.dtype))
        return out.view(-1, 6 * self.hidden)

    def forward(self, temb):
        return self.table(temb).chunk(6, dim=-1)


class AdaLayerNormOut(nn.Module):
    def __init__(self, temb_dim, hidden, eps=1e-6):
        super().__init__()
        self.linear = nn.Linear(temb_dim, 2 * hidden, bias=True)
        self.norm = RMSNormAffine(hidden, eps, affine=False)

    def forward(self, hidden_states, temb, timestep_indices):
        w = self.linear.weight
        shift, scale = self.linear(F.silu(temb.float()).to(w.dtype)).chunk(2, dim=-1)
        h = self.norm(hidden_states)
        return h * (1.0 + scale.index_select(0, timestep_indices)) + shift.index_select(0, timestep_indices)


class H3Block(nn.Module):
    def __init__(self, cfg: H3Config):
        super().__init__()
        D = cfg.hidden_size
        self.norm1 = RMSNormAffine(D, cfg.norm_eps)
        self.norm2 = RMSNormAffine(D, cfg.norm_eps)
        self.adaln_proj = AdaLayerNormModulation(cfg.time_embed_dim, D, cfg.modality_num)
        self.attn = H3Attention(D, cfg.num_attention_heads, cfg.attention_head_dim, cfg.qk_norm_eps)
        self.ff = FeedForward(D, cfg.ff_inner_dim, cfg.ff_activation)

    def forward(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(temb)
        x = hidden_states
        # sm_100a forward + backward kernels for bf16 CUDA rows under autograd, else eager
        normed = adaln_modulated_norm(self.norm1, x, shift_msa, scale_msa, adaln_indices)
        x = x + gate_msa.index_select(0, adaln_indices) * self.attn(normed, rotary_emb, attention_mask)
        normed = adaln_modulated_norm(self.norm2, x, shift_mlp, scale_mlp, adaln_indices)
        return x + gate_mlp.index_select(0, adaln_indices) * self.ff(normed)


class RefinerBlock(nn.Module):
    def __init__(self, cfg: H3Config):
        super().__init__()
        D = cfg.hidden_size
        self.norm1 = RMSNormAffine(D, cfg.norm_eps)
        self.attn = H3Attention(D, cfg.num_attention_heads, cfg.attention_head_dim, cfg.qk_norm_eps)
        self.norm2 = RMSNormAffine(D, cfg.norm_eps)
        self.ff = FeedForward(D, cfg.ff_inner_dim, cfg.ff_activation)

    def forward(self, x):
        x = x + self.attn(self.norm1(x), None)
        return x + self.ff(self.norm2(x))


class TokenRefiner(nn.Module):
    def __init__(self, cfg: H3Config):
        super().__init__()
        self.refiner_blocks = nn.ModuleList([RefinerBlock(cfg) for _ in range(cfg.num_refiner_layers)])

    def forward(self, x):
        for blk in self.refiner_blocks:
            x = blk(x)
        return x


@dataclass
class H3Output:
    sample: torch.Tensor
    audio_sample: torch.Tensor


class H3Transformer(nn.Module):
    """The backbone. `forward` is the eager reference path (training, CPU oracle, teacher);
    inference/engine.py runs the same arithmetic through the fused sm_100a kernels."""

    def __init__(self, cfg: H3Config):
        super().__init__()
        self.config = cfg
        D = cfg.hidden_size
        patch_dim = cfg.in_channels * math.prod(cfg.patch_size)
        self.proj_in = nn.Linear(patch_dim, D)
        self.audio_proj_in = nn.Linear(cfg.audio_in_channels, D)
        self.context_embedder = nn.Linear(cfg.text_dim, D)
        self.token_refiner = TokenRefiner(cfg)
        self.time_proj = Timesteps(cfg.time_freq_dim)
        self.time_embedder = TimestepEmbedding(cfg.time_freq_dim, cfg.time_embed_dim)
        self.rope = RotaryEmbedding3D(cfg.rope_axes_dim, cfg.rope_theta)
        self.transformer_blocks = nn.ModuleList([H3Block(cfg) for _ in range(cfg.num_layers)])
        self.norm_out = AdaLayerNormOut(cfg.time_embed_dim, D, cfg.norm_eps)
        self.proj_out = nn.Linear(D, patch_dim)
        self.audio_proj_out = nn.Linear(D, cfg.audio_in_channels)

    @property
    def dtype(self):
        return self.proj_in.weight.dtype

    def embed(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
              timestep_indices, token_tags, position_ids, video_indices, audio_indices,
              text_indices):
        """Everything before the block stack: packed residual, temb, AdaLN index, rope."""
        dt = self.dtype
        rotary = self.rope(position_ids)
        video = self.proj_in(hidden_states.to(dt))
        audio = self.audio_proj_in(audio_hidden_states.to(dt)) if audio_indices.numel() else None
        text = self.token_refiner(self.context_embedder(encoder_hidden_states.to(dt)))
        S = position_ids.shape[0]
        packed = text.new_zeros((1, S, text.shape[-1]))
        packed = packed.index_copy(1, text_indices, text)
        packed = packed.index_copy(1, video_indices, video.to(text.dtype))
        if audio is not None:
            packed = packed.index_copy(1, audio_indices, audio.to(text.dtype))
        tdt = self.time_embedder.linear_1.weight.dtype
        temb = self.time_embedder(self.time_proj(timestep).to(tdt))
        adaln_indices = timestep_indices * self.config.modality_num + token_tags
        return packed, temb, adaln_indices, rotary

    def head(self, packed, temb, timestep_indices, video_indices, audio_indices):
        packed = self.norm_out(packed, temb, timestep_indices).to(self.proj_out.weight.dtype)
        video_out = self.proj_out(packed).index_select(1, video_indices)
        audio_out = (self.audio_proj_out(packed).index_select(1, audio_indices)
                     if audio_indices.numel() else packed.new_zeros(1, 0, self.config.audio_in_channels))
        return video_out, audio_out

    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                timestep_indices, token_tags, position_ids, video_indices, audio_indices,
                text_indices, attention_kwargs=None, return_dict=True):
        if hidden_states.dim() == 3:
            hidden_states, audio_hidden_states, encoder_hidden_states = (
                hidden_states, audio_hidden_states, encoder_hidden_states)
        packed, temb, adaln_indices, rotary = self.embed(
            hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
            timestep_indices, token_tags, position_ids, video_indices, audio_indices, text_indices)
        for block in self.transformer_blocks:
            packed = block(packed, temb, adaln_indices, rotary)
        video_out, audio_out = self.head(packed, temb, timestep_indices, video_indices, audio_indices)
        if not return_dict:
            return video_out, audio_out
        return H3Output(sample=video_out, audio_sample=audio_out)


def random_init_(model: H3Transformer, seed=0, std=None):
    """Deterministic random init of every parameter in place (the backbone is never
    downloaded here): N(0, 1/fan_in) for matrices, zeros for biases, ones for norm weights
    (apply it to the backbone before the hybrid transform adds its own inits). Runs on
    whatever device the model lives on."""
    g = torch.Generator(device=next(model.parameters()).device).manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() >= 2:
                fan_in = p.shape[1] if p.dim() == 2 else p[0].numel()
                s = std if std is not None else fan_in ** -0.5
                p.copy_(torch.randn(p.shape, generator=g, device=p.device, dtype=torch.float32)
                        .mul_(s).to(p.dtype))
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.fill_(1.0)
    return model
