"""Checkpoint v2: round trips through the .pt and the exploded directory, refusals, key
mapping, ModelSpec validation."""
import os

import pytest
import torch

from vdn_minimax_h3_b200.checkpoints import (CheckpointArtifact, UnsupportedCheckpointFormat,
                                             export_checkpoint_dir, load_checkpoint, save_checkpoint)
from vdn_minimax_h3_b200.checkpoints.key_mapping import map_config, map_key, map_keys
from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID, build_model, load_model_weights, make_spec
from vdn_minimax_h3_b200.models.h3 import h3_tiny_config
from vdn_minimax_h3_b200.models.hybrid_transform import hybrid_new_parameters, transform_config_of_model
from vdn_minimax_h3_b200.models.model_spec import ModelSpec, hybrid_transform_spec


def _artifact(lora=True):
    cfg = h3_tiny_config()
    adapters = []
    if lora:
        from vdn_minimax_h3_b200.models.model_spec import AdapterSpec
        adapters = [AdapterSpec("lora", 1, {"rank": 4, "alpha": 4, "targets": ["attn.orig.to_q"], "name": "default"})]
    spec = make_spec(cfg, RELEASED_HYBRID, adapters=adapters, dtype="float32")
    model = build_model(spec, init="random")
    weights = {n: p.detach().clone() for _, params in hybrid_new_parameters(model) for n, p in params}
    if lora:
        weights["transformer_blocks.0.attn.orig.to_q.lora_A.default.weight"] = torch.randn(4, 256)
        weights["transformer_blocks.0.attn.orig.to_q.lora_B.default.weight"] = torch.randn(256, 4)
    return CheckpointArtifact(kind="weights", model_spec=spec.to_dict(), weights=weights,
                              metadata={"stage": "test"}), model


def test_pt_round_trip(tmp_path):
    art, model = _artifact()
    path = save_checkpoint(art, str(tmp_path / "w.pt"))
    back = load_checkpoint(path)
    assert back.kind == "weights" and back.metadata == {"stage": "test"}
    assert set(back.weights) == set(art.weights)
    fresh = build_model(back.model_spec, init="random", seed=3)
    branch = {k: v for k, v in back.weights.items() if ".lora_" not in k}
    assert load_model_weights(fresh, branch) == len(branch)
    for n, p in fresh.named_parameters():
        if n in branch:
            assert torch.equal(p, branch[n])


def test_dir_round_trip(tmp_path):
    art, _ = _artifact()
    out = export_checkpoint_dir(art, str(tmp_path / "ckpt"), dtype="keep")
    assert os.path.isfile(os.path.join(out, "linear_branch", "model.safetensors"))
    assert os.path.isfile(os.path.join(out, "adapters", "default", "adapter_model.safetensors"))
    back = load_checkpoint(out)
    assert set(back.weights) == set(art.weights)
    for k in art.weights:
        assert torch.equal(back.weights[k], art.weights[k])


def test_refusals(tmp_path):
    torch.save({"kind": "weights", "weights": {}}, tmp_path / "old.pt")
    with pytest.raises(UnsupportedCheckpointFormat):
        load_checkpoint(str(tmp_path / "old.pt"))
    art, _ = _artifact(lora=False)
    art.weights["__window__"] = torch.zeros(1)
    with pytest.raises(UnsupportedCheckpointFormat):
        save_checkpoint(art, str(tmp_path / "bad.pt"))
    bad = CheckpointArtifact(kind="train_state", model_spec=art.model_spec, weights={},
                             optimizer={0: {}}, step=1, rng_state={}, resolved_training_config={})
    with pytest.raises(UnsupportedCheckpointFormat):
        save_checkpoint(bad, str(tmp_path / "bad2.pt"))


def test_key_mapping_and_spec_rules():
    assert map_key("transformer_blocks.3.attn.far.gate.up.weight") == \
        "transformer_blocks.3.attn.linear_attention.output_gate.up.weight"
    assert map_key("transformer_blocks.3.attn.far.alpha.A_log") == \
        "transformer_blocks.3.attn.linear_attention.alpha.A_log"
    assert map_key("transformer_blocks.3.attn.w_o_far.weight") == "transformer_blocks.3.attn.to_out_linear.weight"
    with pytest.raises(ValueError):
        map_keys(["a.attn.far.x", "a.attn.linear_attention.x"])
    flat = map_config({"backend": "vdn_solve", "far_head_dim": 128, "radius": 1, "chunk": 5,
                       "short_conv": "sep", "anchor_frames": True, "w_o_far_scale": 0.5})
    assert flat["short_conv"] == {"targets": ["k", "v"]} and flat["anchor_frames"] == "both"
    assert "w_o_far_scale" not in flat
    t = hybrid_transform_spec({"backend": "vdn_solve", "far_head_dim": 128, "radius": 1,
                               "chunk": 5, "short_conv": "sep", "anchor_frames": True,
                               "bridge": "alpha", "text_state": True, "a_fp32": True})
    assert t.config["softmax_attention"] == {"radius": 1, "chunk": 5}
    spec = make_spec(h3_tiny_config(), RELEASED_HYBRID).to_dict()
    spec["transforms"][0]["config"]["softmax_backend"] = "flex"
    with pytest.raises(ValueError):
        ModelSpec.from_dict(spec)
    spec = make_spec(h3_tiny_config(), RELEASED_HYBRID).to_dict()
    spec["transforms"][0]["config"]["linear_attention"]["linear_head_dim"] = None
    with pytest.raises(ValueError):
        ModelSpec.from_dict(spec)
    spec = make_spec(h3_tiny_config(), RELEASED_HYBRID).to_dict()
    spec["base"]["resolved_config"]["hidden_size"] = 999
    with pytest.raises(ValueError):
        ModelSpec.from_dict(spec)


def test_transform_config_round_trip():
    spec = make_spec(h3_tiny_config(), RELEASED_HYBRID, dtype="float32")
    model = build_model(spec, init="random")
    assert transform_config_of_model(model) == spec.transforms[0].config
