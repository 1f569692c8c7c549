"""Norm, RoPE and window-attention kernels vs fp32 PyTorch references of the same ops."""
import pytest
import torch

from vdn_minimax_h3_b200.models.layout import SequenceLayout
from vdn_minimax_h3_b200.models.window import AttentionPlan, window_bounds, window_softmax_reference
from vdn_minimax_h3_b200.ops import attention as attn_ops
from vdn_minimax_h3_b200.ops import norm as norm_ops
from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,D", [(300, 256), (1000, 5376), (77, 1024)])
def test_adaln_rmsnorm(T, D):
    torch.manual_seed(0)
    x = torch.randn(T, D, device="cuda", dtype=torch.bfloat16) * 3
    w = torch.randn(D, device="cuda")
    table = torch.randn(6, 6 * D, device="cuda", dtype=torch.bfloat16) * 0.2
    idx = torch.randint(0, 6, (T,), device="cuda", dtype=torch.int32)
    out = norm_ops.adaln_rmsnorm(x, w, 1e-6, table, 3 * D, 4 * D, idx)
    check_device_error()
    ref = norm_ops.adaln_rmsnorm_reference(x.cpu(), w.cpu(), 1e-6, table.cpu(), 3 * D, 4 * D, idx.cpu())
    assert _rel(out.cpu(), ref) < 1e-2


def test_frame_sums():
    torch.manual_seed(0)
    x = torch.randn(7 * 100 + 13, 512, device="cuda", dtype=torch.bfloat16)
    out = norm_ops.frame_sums(x, 7, 100, 0, 13)
    ref = x[13:].float().view(7, 100, 512).sum(1)
    assert _rel(out, ref) < 1e-5
    # a shard holding packed rows [250, 480) of the same sequence
    part = norm_ops.frame_sums(x[250:480], 7, 100, 250, 13)
    ref_part = norm_ops.frame_sums(x[250:480].cpu(), 7, 100, 250, 13)
    assert _rel(part, ref_part) < 1e-5


@pytest.mark.parametrize("T,H,d,rot,ld_extra", [(257, 4, 128, 128, 0), (100, 3, 64, 48, 64)])
def test_qk_prep(T, H, d, rot, ld_extra):
    torch.manual_seed(0)
    src_full = torch.randn(T, H * d + ld_extra, device="cuda", dtype=torch.bfloat16)
    src = src_full[:, :H * d]
    w = torch.randn(d, device="cuda")
    ang = torch.randn(T, rot // 2, device="cuda")
    cos = torch.cos(torch.cat([ang, ang], -1)).contiguous()
    sin = torch.sin(torch.cat([ang, ang], -1)).contiguous()
    out = norm_ops.qk_prep(src, H, w, 1e-6, cos, sin)
    ref = norm_ops.qk_prep_reference(src.cpu(), H, w.cpu(), 1e-6, cos.cpu(), sin.cpu())
    assert _rel(out.cpu(), ref) < 1e-2


def _layout(text, audio, F, S):
    return SequenceLayout(seq_len=text + audio + F * S, video_start=text + audio, num_frames=F,
                          tokens_per_frame=S, frame_height=1, frame_width=S, text_start=0,
                          text_len=text)


@pytest.mark.parametrize("text,audio,F,S,H,chunk,radius,anchors", [
    (40, 30, 12, 100, 2, 2, 1, "both"),
    (64, 0, 9, 128, 3, 0, 1, "none"),
    (17, 5, 20, 60, 1, 5, 1, "both"),
])
def test_window_attention_matches_oracle(text, audio, F, S, H, chunk, radius, anchors):
    torch.manual_seed(0)
    lay = _layout(text, audio, F, S)
    bounds = window_bounds(F, radius, chunk)
    plan = AttentionPlan(lay, bounds, anchors, device="cuda")
    T = lay.seq_len
    q = torch.randn(T, H, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    scale = 128 ** -0.5
    out = attn_ops.window_attention(q, k, v, plan, scale)
    check_device_error()
    ref = window_softmax_reference(q.float().cpu(), k.float().cpu(), v.float().cpu(), lay, bounds,
                                   scale, anchors).reshape(T, H * 128)
    assert _rel(out.cpu(), ref) < 2e-2


def test_window_attention_dense_gated_strided():
    torch.manual_seed(1)
    T, H = 1000, 4
    lay = SequenceLayout(seq_len=T, video_start=T, num_frames=0, tokens_per_frame=1)
    plan = AttentionPlan(lay, [], "none", device="cuda", dense=True)
    qkv = torch.randn(T, 3 * H * 128 + 2 * H, device="cuda", dtype=torch.bfloat16) * 2
    q = qkv[:, :H * 128].view(T, H, 128)
    k = qkv[:, H * 128:2 * H * 128].view(T, H, 128)
    v = qkv[:, 2 * H * 128:3 * H * 128].view(T, H, 128)
    gate = qkv[:, 3 * H * 128:3 * H * 128 + H]
    out_full = torch.zeros(T, 2 * H * 128, device="cuda", dtype=torch.bfloat16)
    attn_ops.window_attention(q, k, v, plan, 0.1, gate_logits=gate, out=out_full[:, :H * 128])
    check_device_error()
    ref = attn_ops.window_attention_reference(q.cpu(), k.cpu(), v.cpu(), plan, 0.1, gate.cpu())
    assert _rel(out_full[:, :H * 128].cpu(), ref) < 2e-2
    assert out_full[:, H * 128:].abs().max().item() == 0


@pytest.mark.parametrize("variant,growing", [(0, False), (0, True), (1, True), (2, False),
                                             (3, True), (4, False)])
def test_window_attention_variants(variant, growing):
    """Every exponential-pass variant that computes the attention (scalar, packed f32x2, and
    the packed pass with 2/16, 4/16 or 6/16 of the exponentials on the polynomial) matches
    the oracle like the default instance. `growing` scales the keys up along the sequence so
    later blocks raise the running max by more than 2^8 and the O rescale path runs. The
    timing-only variants 5-7 compute wrong results on purpose and are not checked."""
    from vdn_minimax_h3_b200.ops._ext import ext
    torch.manual_seed(2)
    lay = _layout(40, 30, 12, 100)
    bounds = window_bounds(12, 1, 2)
    plan = AttentionPlan(lay, bounds, "both", device="cuda")
    T = lay.seq_len
    q = torch.randn(T, 2, 128, device="cuda", dtype=torch.bfloat16) * 2
    k, v = torch.randn_like(q), torch.randn_like(q)
    if growing:
        ramp = torch.linspace(0.5, 6.0, T, device="cuda").view(T, 1, 1)
        k = (k.float() * ramp).to(torch.bfloat16)
    prev = ext().attention_variant()
    ext().attention_set_variant(variant)
    try:
        out = attn_ops.window_attention(q, k, v, plan, 128 ** -0.5)
        check_device_error()
    finally:
        ext().attention_set_variant(prev)
    ref = window_softmax_reference(q.float().cpu(), k.float().cpu(), v.float().cpu(), lay, bounds,
                                   128 ** -0.5, "both").reshape(T, 2 * 128)
    assert _rel(out.cpu(), ref) < 2e-2
