"""CPU: the inference engine's packed/fused block equals the eager reference forward, the
tiny golden sampling run (the 2-block CPU configuration), and the full-cover == dense-teacher rule."""
import copy

import pytest
import torch

from vdn_minimax_h3_b200.inference.engine import InferenceEngine
from vdn_minimax_h3_b200.inference.render import build_inputs, generate_latents, render_geometry
from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID, TINY_HYBRID, build_model, make_spec
from vdn_minimax_h3_b200.models.h3 import H3Config, h3_tiny_config
from vdn_minimax_h3_b200.models.hybrid_transform import iter_hybrids, set_layout, set_teacher_mode


def tiny_model(hybrid=TINY_HYBRID, cfg=None, seed=0):
    torch.manual_seed(seed)
    cfg = cfg or h3_tiny_config()
    spec = make_spec(cfg, hybrid, dtype="float32")
    return build_model(spec, init="random", seed=seed)


def _forward_inputs(cfg, geo, text_len, seed=0):
    packed, layout, idx = build_inputs(geo, text_len, "cpu")
    g = torch.Generator().manual_seed(seed)
    nv = idx["video_indices"].numel()
    patch_dim = cfg.in_channels * 4
    kw = dict(hidden_states=torch.randn(1, nv, patch_dim, generator=g),
              audio_hidden_states=torch.randn(1, idx["audio_indices"].numel(), 32, generator=g),
              encoder_hidden_states=torch.randn(1, text_len, cfg.text_dim, generator=g),
              token_tags=idx["token_tags"], position_ids=idx["position_ids"],
              video_indices=idx["video_indices"], audio_indices=idx["audio_indices"],
              text_indices=idx["text_indices"], return_dict=False)
    S = idx["position_ids"].shape[0]
    row_t = torch.full((S,), 0.25)
    if idx["audio_indices"].numel():
        row_t[idx["audio_indices"]] = 0.6
    kw["timestep"], kw["timestep_indices"] = torch.unique(row_t, sorted=True, return_inverse=True)
    return kw, layout


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


@torch.no_grad()
def test_engine_matches_eager_tiny():
    cfg = h3_tiny_config()
    model = tiny_model()
    geo = render_geometry(cfg, 5, latent_h=16, latent_w=16, audio=False, num_latent_frames=4)
    kw, layout = _forward_inputs(cfg, geo, 32)
    set_layout(model, layout)
    ref_v, _ = model(**kw)
    eng = InferenceEngine(copy.deepcopy(model))
    out_v, _ = eng(**kw, layout=layout)
    assert _rel(out_v, ref_v) < 1e-4


@torch.no_grad()
def test_engine_matches_eager_released_transform():
    """c1 window, anchors both, vdn_solve, K/V short conv, text state, audio rows."""
    cfg = H3Config(hidden_size=128, num_layers=2, num_attention_heads=2, attention_head_dim=64,
                   in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                   ff_inner_dim=256, num_refiner_layers=1, rope_axes_dim=(16, 24, 24))
    model = tiny_model(RELEASED_HYBRID, cfg)
    geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=17)
    geo.num_audio_latents = 6
    kw, layout = _forward_inputs(cfg, geo, 10)
    set_layout(model, layout)
    ref_v, ref_a = model(**kw)
    eng = InferenceEngine(copy.deepcopy(model))
    out_v, out_a = eng(**kw, layout=layout)
    assert _rel(out_v, ref_v) < 1e-4
    assert _rel(out_a, ref_a) < 1e-4


@torch.no_grad()
def test_full_cover_hybrid_equals_teacher():
    cfg = h3_tiny_config()
    hy = copy.deepcopy(TINY_HYBRID)
    hy["softmax_attention"] = dict(radius=10, chunk=0)
    model = tiny_model(hy)
    # zero the softmax gate's bias effect: full cover still applies the 0.99 gate, so
    # compare against the teacher with the gate folded in via teacher_mode off/on outputs.
    for attn in iter_hybrids(model):
        attn.enable_softmax_gate = False
    geo = render_geometry(cfg, 5, latent_h=16, latent_w=16, audio=False, num_latent_frames=4)
    kw, layout = _forward_inputs(cfg, geo, 32)
    set_layout(model, layout)
    hyb, _ = model(**kw)
    set_teacher_mode(model, True)
    teach, _ = model(**kw)
    assert _rel(hyb, teach) < 1e-5


@torch.no_grad()
def test_tiny_golden_two_euler_steps():
    """The tiny CPU configuration: latent [1,16,4,16,16], text [1,32,256], 2 Euler steps at sigma
    1.0 and 0.5 (shift 1); engine and eager agree and the run is deterministic."""
    cfg = h3_tiny_config()
    model = tiny_model()
    emb = torch.randn(32, 256, generator=torch.Generator().manual_seed(1))

    def run(m):
        return generate_latents(m, emb, 5, 2, seed=7, device="cpu", model_config=cfg,
                                video_shift=1.0, audio_shift=1.0, latent_h=16, latent_w=16,
                                audio=False, num_latent_frames=4,
                                on_layout=lambda lay: set_layout(model, lay))

    lat1, _ = run(model)
    lat2, _ = run(model)
    assert lat1.shape == (1, 16, 4, 16, 16)
    assert torch.isfinite(lat1).all()
    assert torch.equal(lat1, lat2)
    eng = InferenceEngine(copy.deepcopy(model))
    set_layout(eng.model, None)
    lat3, _ = generate_latents(eng, emb, 5, 2, seed=7, device="cpu", model_config=cfg,
                               video_shift=1.0, audio_shift=1.0, latent_h=16, latent_w=16,
                               audio=False, num_latent_frames=4,
                               on_layout=lambda lay: set_layout(eng.model, lay))
    assert _rel(lat3, lat1) < 1e-4


def test_column_route_cpu_semantics():
    """ColumnRoute on CPU: raw planes copy columns, plane 1 of q/k heads gets QK-prep."""
    from vdn_minimax_h3_b200.ops import gemm
    from vdn_minimax_h3_b200.ops.norm import qk_prep_reference
    from vdn_minimax_h3_b200.models.h3 import RotaryEmbedding3D
    torch.manual_seed(0)
    M, K, N = 40, 64, 272
    x, w = torch.randn(M, K), torch.randn(N, K) / 8
    pos = torch.stack([torch.arange(M) // 10, torch.arange(M) % 5, torch.arange(M) % 3], 1)
    cos, sin = RotaryEmbedding3D((32, 48, 48))(pos)
    raw, q, rep = torch.zeros(M, N), torch.zeros(M, 128), torch.zeros(M, 16)
    route = gemm.ColumnRoute(N, planes=3)
    route.place(0, raw).place(0, q, plane=1).place(256, rep, plane=2)
    nq = torch.rand(128) + 0.5
    gemm.linear_routed(x, w, None, route, (0, 128), (0, 0), nq, None, 1e-6, cos, sin)
    y = x @ w.t()
    assert torch.allclose(raw, y, atol=1e-5)
    assert torch.allclose(rep, y[:, 256:272], atol=1e-5)
    assert torch.allclose(q, qk_prep_reference(y[:, :128], 1, nq, 1e-6, cos, sin), atol=1e-5)
    with pytest.raises(ValueError):
        route.place(4, raw[:, :8])
