"""The prompt cache: the `.pt` every render reads (reference src/inference/utils/
prompt_cache.py:12-38).

    prompt, prompt_embeds (L, 5120) bf16, text_token_tags (L,)        every cache
    keyframe_anchors, condition_latents [(1, 24, 1, h, w) fp32 ...]    keyframes or references

Anchors: ("first",) i2va, ("last",) l2va, ("first", "last") fl2va, all "ref" = ref2va.
`synthetic_prompt` makes a cache of random embeddings (no text encoder offline).
"""
import os

import torch

REFERENCE_ANCHOR = "ref"
KEYFRAME_MODES = {("first",): "i2va", ("last",): "l2va", ("first", "last"): "fl2va"}


def is_reference_request(anchors):
    return bool(anchors) and all(a == REFERENCE_ANCHOR for a in anchors)


def conditioning_mode(anchors):
    if not anchors:
        return "t2va"
    if is_reference_request(anchors):
        return "ref2va"
    return KEYFRAME_MODES[tuple(anchors)]


def load_prompt(prompt_file, device):
    """-> (prompt_embeds bf16 [L, D], text_token_tags [L], conditions or None)."""
    data = torch.load(prompt_file, map_location="cpu", weights_only=True)
    conditions = None
    if data.get("keyframe_anchors"):
        conditions = (tuple(data["keyframe_anchors"]),
                      [c.to(device, torch.float32) for c in data["condition_latents"]])
    return data["prompt_embeds"].to(device, torch.bfloat16), data["text_token_tags"], conditions


def save_prompt(path, prompt, prompt_embeds, text_token_tags=None, keyframe_anchors=(),
                condition_latents=(), **extra):
    """Atomic write (.tmp then rename). `extra` carries the keyframe encoder's
    keyframe_files / height / width / reference_size fields."""
    if text_token_tags is None:
        text_token_tags = torch.ones(prompt_embeds.shape[0], dtype=torch.long)
    payload = {"prompt": prompt, "prompt_embeds": prompt_embeds.to(torch.bfloat16).cpu(),
               "text_token_tags": torch.as_tensor(text_token_tags, dtype=torch.long).cpu()}
    if keyframe_anchors:
        payload["keyframe_anchors"] = list(keyframe_anchors)
        payload["condition_latents"] = [c.float().cpu() for c in condition_latents]
    payload.update(extra)
    tmp = path + ".tmp"
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    torch.save(payload, tmp)
    os.replace(tmp, path)
    return path


def synthetic_prompt(length=800, width=5120, seed=0, anchors=(), latent_hw=(48, 84), channels=24):
    g = torch.Generator().manual_seed(seed)
    emb = torch.randn(length, width, generator=g).to(torch.bfloat16)
    conds = [torch.randn(1, channels, 1, *latent_hw, generator=g) for _ in anchors]
    return {"prompt": "<synthetic>", "prompt_embeds": emb,
            "text_token_tags": torch.ones(length, dtype=torch.long),
            "keyframe_anchors": list(anchors), "condition_latents": conds}
