"""The Stage-DMD adapter pair: the external few-step ("turbo") LoRA as a live, trainable
adapter and the fake score's adapter over the same targets.

Reference parity: src/training/turbo_adapter.py:17-151. The external checkpoint is read
and translated by `inference.lora.load_external_lora`; its dense attention targets are
re-rooted through HybridAttention's `attn.orig`; the adapter config (AdapterSpec form:
default rank = the most common rank, per-module `rank_pattern` / `alpha_pattern` for the
rest, alpha == rank so the update is exactly B @ A) is derived from the tensors; the fake
adapter takes the same exact target set at one uniform rank with B = 0 (so the fake score
equals the real score at step 0). Adapters are `models.lora.LoraLinear` layers with peft's
key naming (`<module>.lora_A.<adapter>.weight`); switching the active set never touches
requires_grad (FSDP2 owns those flags after sharding).
"""
from collections import Counter

from torch import nn

from vdn_minimax_h3_b200.models.lora import LoraLinear, set_active_adapters  # noqa: F401

BLOCK_PREFIXES = ("transformer_blocks.", "token_refiner.refiner_blocks.")


def reroot_external_lora_state(model, state):
    """Resolve each LoRA key's module against the hybrid model: a dense `.attn.` target
    that only exists under the HybridAttention wrapper moves to `.attn.orig.`. Values are
    untouched; unknown modules and non-LoRA keys are refused."""
    modules = dict(model.named_modules())
    out = {}
    for key, tensor in state.items():
        marker = ".lora_A." if ".lora_A." in key else ".lora_B." if ".lora_B." in key else None
        if marker is None:
            raise ValueError(f"external adapter state has a non-LoRA key: {key}")
        target, suffix = key.split(marker, 1)
        tried = [target] + ([target.replace(".attn.", ".attn.orig.", 1)] if ".attn." in target else [])
        found = next((t for t in tried if t in modules), None)
        if found is None:
            raise KeyError(f"adapter target {target!r} has no module; tried {tried}")
        out[found + marker + suffix] = tensor
    return out


def adapter_config_from_state(state, name="turbo"):
    """AdapterSpec-form config of a (re-rooted) LoRA state: exact targets, the most common
    rank as default, the others in rank_pattern (alpha_pattern equal: alpha == rank)."""
    ranks = {key.split(".lora_A.", 1)[0]: int(t.shape[0])
             for key, t in state.items() if ".lora_A." in key}
    if not ranks:
        raise ValueError("adapter state has no lora_A tensors")
    default = Counter(ranks.values()).most_common(1)[0][0]
    pattern = dict(sorted((k, r) for k, r in ranks.items() if r != default))
    return {"name": name, "rank": default, "alpha": default, "targets": sorted(ranks),
            "rank_pattern": pattern, "alpha_pattern": dict(pattern), "exact_targets": True}


def extra_shard_module_paths(config):
    """Adapter targets outside the two block stacks (e.g. norm_out.linear): Stage DMD must
    shard these explicitly, the block sharder does not own them."""
    return sorted({t for t in config["targets"] if not t.startswith(BLOCK_PREFIXES)})


def fake_adapter_config(turbo_config, rank, name="fake"):
    """The fake score's adapter: the turbo adapter's exact targets at one uniform rank,
    alpha == rank."""
    if rank < 1:
        raise ValueError(f"fake adapter rank must be >= 1, got {rank}")
    return {"name": name, "rank": int(rank), "alpha": int(rank),
            "targets": list(turbo_config["targets"]), "rank_pattern": {}, "alpha_pattern": {},
            "exact_targets": True}


def load_external_adapter(model, checkpoint, name="turbo"):
    """(re-rooted state, config) of an external LoRA file; scaled variants are refused."""
    from vdn_minimax_h3_b200.inference.lora import load_external_lora
    state, scale, _ = load_external_lora(checkpoint)
    if scale != 1.0:
        raise ValueError(f"Stage DMD expects a unit LoRA scale (alpha == rank), got {scale}")
    state = reroot_external_lora_state(model, state)
    return state, adapter_config_from_state(state, name)


def inject_lora_adapter(model, config, adapter_name=None):
    """Wrap exactly the config's target Linears (module paths) with one named adapter at
    the per-module rank / alpha. -> number of wrapped layers."""
    name = adapter_name or config["name"]
    targets = set(config["targets"])
    ranks, alphas = config.get("rank_pattern", {}), config.get("alpha_pattern", {})
    seen = set()
    for mod_name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            full = f"{mod_name}.{child_name}" if mod_name else child_name
            if full not in targets:
                continue
            if not isinstance(child, (nn.Linear, LoraLinear)):
                raise TypeError(f"adapter target {full} is a {type(child).__name__}, not Linear")
            lin = child if isinstance(child, LoraLinear) else LoraLinear(child)
            lin.add_adapter(name, int(ranks.get(full, config["rank"])),
                            float(alphas.get(full, config["alpha"])))
            setattr(module, child_name, lin)
            seen.add(full)
    missing = targets - seen
    if missing:
        raise KeyError(f"adapter targets without a module: {sorted(missing)[:4]}")
    return len(seen)


def copy_adapter_state(model, state, adapter_name):
    """Copy `<module>.lora_[AB].weight` tensors into the named adapter's parameters."""
    params = dict(model.named_parameters())
    copied = 0
    for key, tensor in state.items():
        for marker in (".lora_A.", ".lora_B."):
            if marker in key:
                target = key.replace(marker, f"{marker}{adapter_name}.")
                break
        else:
            raise ValueError(f"not a LoRA tensor: {key}")
        if target not in params:
            raise KeyError(f"the injected adapter has no parameter {target}")
        if params[target].shape != tensor.shape:
            raise ValueError(f"shape mismatch for {target}: {tuple(params[target].shape)} vs "
                             f"{tuple(tensor.shape)}")
        params[target].data.copy_(tensor.to(params[target].dtype))
        copied += 1
    return copied


def is_named_adapter_parameter(name, adapter_name):
    return f".lora_A.{adapter_name}." in name or f".lora_B.{adapter_name}." in name
