"""Stage-DMD adapter handling: re-rooting an external LoRA through HybridAttention's
`attn.orig`, the mixed-rank AdapterSpec config, injection + copy reproducing W + B A, the
fake adapter (B = 0, same targets) and active-set switching without requires_grad edits."""
import pytest
import torch

from tests.test_model_cpu import tiny_model
from vdn_minimax_h3_b200.models.lora import set_active_adapters
from vdn_minimax_h3_b200.training import turbo_adapter as ta


def _external_state(model, ranks=(4, 4, 2)):
    """Dense-layout keys (no `.orig`): what an external few-step adapter ships."""
    g = torch.Generator().manual_seed(3)
    state = {}
    for i, _ in enumerate(model.transformer_blocks):
        for t, r in zip(("to_q", "to_k", "to_v"), ranks):
            lin = model.get_submodule(f"transformer_blocks.{i}.attn.orig.{t}")
            state[f"transformer_blocks.{i}.attn.{t}.lora_A.weight"] = torch.randn(r, lin.in_features, generator=g) * 0.1
            state[f"transformer_blocks.{i}.attn.{t}.lora_B.weight"] = torch.randn(lin.out_features, r, generator=g) * 0.1
    return state


def test_reroot_config_inject_copy():
    model = tiny_model()
    ext = _external_state(model)
    state = ta.reroot_external_lora_state(model, ext)
    assert all(".attn.orig." in k for k in state)
    cfg = ta.adapter_config_from_state(state, "turbo")
    assert cfg["rank"] == 4 and cfg["alpha"] == 4 and cfg["exact_targets"]
    assert set(cfg["rank_pattern"].values()) == {2} and cfg["rank_pattern"] == cfg["alpha_pattern"]
    assert ta.extra_shard_module_paths(cfg) == []
    key = "transformer_blocks.0.attn.orig.to_v"
    base = model.get_submodule(key).weight.detach().clone()
    n = ta.inject_lora_adapter(model, cfg)
    assert n == len(cfg["targets"])
    assert ta.copy_adapter_state(model, state, "turbo") == len(state)
    lin = model.get_submodule(key)
    x = torch.randn(3, lin.in_features)
    want = x @ (base + state[key + ".lora_B.weight"] @ state[key + ".lora_A.weight"]).t()
    if lin.bias is not None:
        want = want + lin.bias
    torch.testing.assert_close(lin(x), want, rtol=1e-4, atol=1e-4)

    fake = ta.fake_adapter_config(cfg, 8)
    assert fake["targets"] == cfg["targets"] and fake["rank_pattern"] == {}
    ta.inject_lora_adapter(model, fake)
    assert lin.lora_A["fake"].weight.shape[0] == 8
    assert torch.count_nonzero(lin.lora_B["fake"].weight) == 0     # fake == real at step 0
    flags = {n: p.requires_grad for n, p in model.named_parameters()}
    set_active_adapters(model, ["fake"])
    torch.testing.assert_close(lin(x), x @ base.t() + (lin.bias if lin.bias is not None else 0),
                               rtol=1e-4, atol=1e-4)
    assert flags == {n: p.requires_grad for n, p in model.named_parameters()}
    names = [n for n, _ in model.named_parameters() if ta.is_named_adapter_parameter(n, "turbo")]
    assert len(names) == 2 * len(cfg["targets"])


def test_refusals():
    model = tiny_model()
    with pytest.raises(ValueError):
        ta.reroot_external_lora_state(model, {"transformer_blocks.0.attn.to_q.weight": torch.zeros(1)})
    with pytest.raises(KeyError):
        ta.reroot_external_lora_state(model, {"nope.lora_A.weight": torch.zeros(1, 1)})
    with pytest.raises(ValueError):
        ta.fake_adapter_config({"targets": []}, 0)
