"""The portable component render on a B200: the exported component's eager bf16 transformer
with its DiT blocks streamed from pinned host memory (--offload_dit) samples the same
latents as the resident transformer, and a clip is written as one mp4 with sound."""
import os

import pytest
import torch

from tests.test_infer_component_cpu import _component
from vdn_minimax_h3_b200.inference import infer_component, mp4mux
from vdn_minimax_h3_b200.inference.render import generate_latents

pytestmark = pytest.mark.gpu


def test_streamed_blocks_match_resident_on_gpu(tmp_path):
    comp = _component(tmp_path)
    dev = torch.device("cuda")
    emb = torch.randn(12, 256, generator=torch.Generator().manual_seed(0)).to(dev, torch.bfloat16)
    outs = []
    for offload in (False, True):
        mod, model = infer_component.load_transformer(comp, random_base_seed=3)
        model, streamer = infer_component.place(model, dev, offload_dit=offload)
        outs.append(generate_latents(model, emb, 5, 2, 0, dev, model.config, latent_h=8,
                                     latent_w=8, on_layout=lambda lay, m=model: mod.set_layout(m, lay)))
        if offload:
            assert streamer.host_bytes() > 0
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)


def test_component_render_on_gpu(tmp_path):
    comp = _component(tmp_path)
    out = str(tmp_path / "clip.mp4")
    rec = infer_component.render(comp, "a quiet harbour at dawn", out=out, steps=2, frames=5,
                                 random_base_seed=3, device="cuda", latent_hw=(8, 8),
                                 offload_dit=True)
    assert os.path.getsize(out) > 0 and rec["frames"] == 5
    with open(out, "rb") as f:
        assert sorted(mp4mux.track_handlers(f.read())) == [b"soun", b"vide"]
