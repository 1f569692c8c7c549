"""Block-streamed inference on a B200: the fused-kernel engine with its blocks streamed from
pinned host memory (side-stream prefetch) matches the resident engine, two model evaluations
in a row, and leaves only the prefetched block on the device."""
import copy

import pytest
import torch

from vdn_minimax_h3_b200.ops._ext import check_device_error

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@torch.no_grad()
def test_block_offload_on_gpu():
    from tests.test_model_cpu import _forward_inputs, tiny_model
    from vdn_minimax_h3_b200.inference.engine import InferenceEngine
    from vdn_minimax_h3_b200.inference.offload import enable_block_offload
    from vdn_minimax_h3_b200.inference.render import render_geometry
    from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID
    from vdn_minimax_h3_b200.models.h3 import H3Config
    from vdn_minimax_h3_b200.models.hybrid_transform import set_layout
    cfg = H3Config(hidden_size=256, num_layers=3, num_attention_heads=2, attention_head_dim=128,
                   in_channels=8, text_dim=96, time_embed_dim=64, time_freq_dim=32,
                   ff_inner_dim=512, num_refiner_layers=1, rope_axes_dim=(32, 48, 48))
    model = tiny_model(RELEASED_HYBRID, cfg)
    geo = render_geometry(cfg, 5, latent_h=8, latent_w=12, audio=True, num_latent_frames=17)
    geo.num_audio_latents = 6
    kw, layout = _forward_inputs(cfg, geo, 24)
    set_layout(model, layout)
    kwg = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in kw.items()}

    def gpu_model():
        m = copy.deepcopy(model).to(device="cuda", dtype=torch.bfloat16)
        m.time_embedder.float()
        for blk in m.transformer_blocks:
            blk.attn.linear_attention.alpha.float()
        return m

    ref, _ = InferenceEngine(gpu_model())(**kwg, layout=layout)
    eng = InferenceEngine(gpu_model())
    streamer = enable_block_offload(eng)
    assert all(g[0].is_pinned() for b in streamer.blocks for g in b.groups.values())
    for _ in range(2):
        out, _ = eng(**kwg, layout=layout)
        torch.cuda.synchronize()
        check_device_error()
        assert _rel(out, ref) < 1e-3
    assert [b.resident for b in streamer.blocks] == [True, False, False]
