"""The portable component render: an exported component directory is imported on its own,
its eager transformer samples a clip and the clip is written as one mp4 with sound; the
block-streamed placement (--offload_dit) gives the same latents as the resident one."""
import os

import torch

from tests.test_checkpoints import _artifact
from vdn_minimax_h3_b200.checkpoints import export_checkpoint_dir
from vdn_minimax_h3_b200.export import component
from vdn_minimax_h3_b200.inference import infer_component, mp4mux
from vdn_minimax_h3_b200.inference.render import generate_latents


def _component(tmp_path):
    art, _ = _artifact()
    ckpt = export_checkpoint_dir(art, str(tmp_path / "ckpt"), dtype="keep")
    out_dir, _ = component.export_component(ckpt)
    return out_dir


def test_component_render_writes_mp4_with_sound(tmp_path):
    comp = _component(tmp_path)
    out = str(tmp_path / "clip.mp4")
    rec = infer_component.render(comp, "a quiet harbour at dawn", out=out, steps=2, frames=5,
                                 random_base_seed=3, device="cpu", latent_hw=(8, 8))
    assert rec["out"] == out and os.path.getsize(out) > 0
    assert rec["frames"] == 5 and len(rec["step_seconds"]) == 2
    with open(out, "rb") as f:
        handlers = mp4mux.track_handlers(f.read())
    assert sorted(handlers) == [b"soun", b"vide"]


def test_offloaded_blocks_match_resident(tmp_path):
    comp = _component(tmp_path)
    mod, model = infer_component.load_transformer(comp, random_base_seed=3, dtype=torch.float32)
    emb = torch.randn(12, model.config.text_dim)

    def sample(m):
        return generate_latents(m, emb, 5, 2, 0, torch.device("cpu"), m.config, latent_h=8,
                                latent_w=8, on_layout=lambda lay: mod.set_layout(m, lay))

    want = sample(model)
    _, model2 = infer_component.load_transformer(comp, random_base_seed=3, dtype=torch.float32)
    model2, streamer = infer_component.place(model2, torch.device("cpu"), offload_dit=True)
    assert streamer is not None and streamer.host_bytes() > 0
    got = sample(model2)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    # between evaluations only block 0 is resident (prefetched for the next evaluation)
    assert [b.resident for b in streamer.blocks] == [True] + [False] * (len(streamer.blocks) - 1)
