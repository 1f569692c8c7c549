"""LoRA merging at load: W += scale * (B @ A), the delta in fp32, added in the weight's dtype.

Reference parity: src/inference/utils/lora.py:32-117 -- the checkpoint's own adapters and
external (community) adapters merge the same way; a dense-model target name is re-rooted
through `.attn.orig.` on a hybrid; external files may carry alpha in their metadata
(scale = alpha / rank); original-layout adapters (fused qkv_proj, mlp.fc1 with [gate; value]
halves) are translated onto the diffusers names.
"""
import re

import torch

_ORIGINAL_RENAMES = ((".mlp.fc1.", ".ff.net.0.proj."), (".mlp.fc2.", ".ff.net.2."),
                     (".attn.out_proj.", ".attn.to_out.0."))


def translate_original_layout(state):
    """Original-layout keys (blocks.N..., fused qkv_proj, fc1 [gate; value]) -> diffusers
    names with [value; gate] and per-projection q/k/v pairs. Diffusers-named state passes."""
    if not any(".qkv_proj." in k for k in state):
        return state
    out = {}
    for name, t in state.items():
        if name.startswith("diffusion_model."):
            name = name[len("diffusion_model."):]
        name = re.sub(r"^blocks\.", "transformer_blocks.", name)
        name = name.replace("token_refiner.blocks.", "token_refiner.refiner_blocks.")
        name = name.replace("final_layer.adaln_proj.linear.", "norm_out.linear.")
        if ".mlp.fc1." in name and ".lora_B." in name:
            gate, value = t.chunk(2, dim=0)
            t = torch.cat([value, gate], dim=0)
        for old, new in _ORIGINAL_RENAMES:
            name = name.replace(old, new)
        if ".attn.qkv_proj." in name:
            parts = (t, t, t) if ".lora_A." in name else t.chunk(3, dim=0)
            for proj, part in zip(("to_q", "to_k", "to_v"), parts):
                out[name.replace(".attn.qkv_proj.", f".attn.{proj}.")] = part
            continue
        out[name] = t
    return out


def resolve_target(params, target):
    if target in params:
        return params[target]
    if ".attn." in target:
        rerooted = target.replace(".attn.", ".attn.orig.", 1)
        if rerooted in params:
            return params[rerooted]
    raise KeyError(f"LoRA target {target!r} has no parameter (also tried the .attn.orig. re-root)")


@torch.no_grad()
def merge_lora_state(model, state, scale=1.0):
    """Fold peft-named `.lora_A.` / `.lora_B.` pairs into the model in place; returns the
    number of pairs merged. Names may carry the adapter infix (`.lora_A.default.weight`)."""
    params = dict(model.named_parameters())
    merged = 0
    for name, a in state.items():
        if ".lora_A." not in name:
            continue
        b = state[name.replace(".lora_A.", ".lora_B.")]
        target = name.split(".lora_A.")[0] + ".weight"
        w = resolve_target(params, target)
        delta = (b.to(w.device, torch.float32) @ a.to(w.device, torch.float32)) * scale
        w.add_(delta.to(w.dtype))
        merged += 1
    return merged


def load_external_lora(path, alpha=None):
    """A community LoRA safetensors -> (state, scale, ranks); `.default.` infix stripped."""
    from safetensors import safe_open
    state = {}
    with safe_open(path, framework="pt") as f:
        meta = f.metadata() or {}
        for key in f.keys():
            state[key.replace(".default.", ".")] = f.get_tensor(key)
    state = translate_original_layout(state)
    ranks = sorted({state[k].shape[0] for k in state if ".lora_A." in k})
    if alpha is None and "alpha" not in meta:
        return state, 1.0, ranks
    if len(ranks) != 1:
        raise ValueError(f"{path}: one alpha cannot scale mixed ranks {ranks}")
    alpha = float(meta["alpha"]) if alpha is None else float(alpha)
    return state, alpha / ranks[0], ranks


def random_lora_state(model, rank, targets=("to_q", "to_k", "to_v", "to_out.0"), seed=0,
                      name="default", std=0.02, device=None):
    """A synthetic peft-named adapter over every DiT block's attention projections (the
    bench's stand-in for the Stage-B `default` / Stage-DMD `turbo` adapters)."""
    g = torch.Generator(device=device or "cpu").manual_seed(seed)
    state = {}
    for i, blk in enumerate(model.transformer_blocks):
        attn = blk.attn.orig if hasattr(blk.attn, "orig") else blk.attn
        for t in targets:
            lin = attn.to_out[0] if t == "to_out.0" else getattr(attn, t)
            out_f, in_f = lin.weight.shape
            pre = f"transformer_blocks.{i}.attn.{t}"
            state[f"{pre}.lora_A.{name}.weight"] = torch.randn(rank, in_f, generator=g, device=device) * std
            state[f"{pre}.lora_B.{name}.weight"] = torch.randn(out_f, rank, generator=g, device=device) * std
    return state
