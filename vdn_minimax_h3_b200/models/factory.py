"""build_model(spec): the one constructor every stage uses.

Reference parity: src/models/factory.py:30-153 (load the base named by the spec, verify
its config against the spec's resolved_config, apply the transforms; adapters are NOT
injected here; load_model_weights is strict).

The base named `diffusers / MiniMaxH3Transformer3DModel` (the reference's stamp) maps to
this package's H3Transformer, whose parameter tree uses the same names. Base weights come
from `source` when it is a directory of safetensors shards; with `init="random"` (or
VDN_SYNTHETIC_BASE semantics in the bench) the backbone is random-initialised instead --
no network, no download.
"""
import glob
import json
import os
from typing import Any, Dict, Optional, Union

import torch

from vdn_minimax_h3_b200.models.h3 import H3Config, H3Transformer, random_init_
from vdn_minimax_h3_b200.models.hybrid_transform import (TRANSFORM_TYPE,
                                                         apply_hybrid_attention_transform)
from vdn_minimax_h3_b200.models.model_spec import (HYBRID_TRANSFORM_VERSION, BaseSpec, ModelSpec,
                                                   TransformSpec, validate_spec)

KNOWN_BASES = {("diffusers", "MiniMaxH3Transformer3DModel"), ("vdn_minimax_h3_b200", "H3Transformer")}
_TRANSFORMS = {TRANSFORM_TYPE: apply_hybrid_attention_transform}
DTYPES = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}
CONFIG_KEYS = ("hidden_size", "num_layers", "num_attention_heads", "attention_head_dim")


def h3_config_from_resolved(resolved: Dict[str, Any]) -> H3Config:
    return H3Config.from_dict({k: v for k, v in resolved.items() if not k.startswith("_")})


def empty_model(cfg: H3Config, device="cpu", dtype=torch.bfloat16):
    """The backbone with uninitialised storage on `device` in `dtype` (time embedder fp32)."""
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device("meta"):
            model = H3Transformer(cfg)
    finally:
        torch.set_default_dtype(prev)
    model = model.to_empty(device=device)
    model.time_embedder.float()
    return model


def load_base_weights(model, source, subfolder="transformer"):
    """Copy every tensor of the safetensors shards under source/subfolder into the model."""
    from safetensors import safe_open
    root = os.path.join(source, subfolder) if subfolder else source
    files = sorted(glob.glob(os.path.join(root, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no safetensors under {root}")
    params = dict(model.named_parameters())
    seen = 0
    with torch.no_grad():
        for f in files:
            with safe_open(f, framework="pt") as h:
                for key in h.keys():
                    if key in params:
                        p = params[key]
                        p.copy_(h.get_tensor(key).to(device=p.device, dtype=p.dtype))
                        seen += 1
    missing = len(params) - seen
    if missing:
        raise RuntimeError(f"{missing} base parameters were not found under {root}")
    return seen


def build_model(spec: Union[ModelSpec, Dict[str, Any]], device="cpu", base_source=None,
                init: str = "load", seed: int = 0):
    """spec -> canonical model (base + transforms, no adapters, no overlays).

    init="load": base weights from `base_source or spec.base.source` (safetensors shards).
    init="random": deterministic random backbone (synthetic runs; nothing downloaded)."""
    if not isinstance(spec, ModelSpec):
        spec = ModelSpec.from_dict(spec)
    validate_spec(spec)
    base = spec.base
    if (base.library, base.class_name) not in KNOWN_BASES:
        raise ValueError(f"unknown base {base.library}.{base.class_name}")
    cfg = h3_config_from_resolved(base.resolved_config)
    dtype = DTYPES[base.resolved_config.get("_load_dtype", "bfloat16")]
    model = empty_model(cfg, device=device, dtype=dtype)
    if init == "random":
        random_init_(model, seed=seed)
    elif init == "load":
        from vdn_minimax_h3_b200.paths import resolve_weights
        load_base_weights(model, resolve_weights(base_source or base.source), base.subfolder)
    else:
        raise ValueError(f"init must be 'load' or 'random', got {init!r}")
    verify_base_config(model, base)
    for t in spec.transforms:
        if t.type not in _TRANSFORMS:
            raise ValueError(f"unknown transform {t.type!r} (version {t.version})")
        _TRANSFORMS[t.type](model, t.config)
    return model


def verify_base_config(model, base: BaseSpec):
    live = model.config.to_dict()
    for key, want in base.resolved_config.items():
        if key.startswith("_"):
            continue
        if key in live and live[key] != want and not (
                isinstance(want, list) and list(live[key]) == want):
            raise ValueError(f"base config mismatch on {key!r}: spec says {want!r}, "
                             f"model says {live[key]!r}")


def make_spec(cfg: H3Config, hybrid: Optional[Dict[str, Any]] = None, source="synthetic",
              adapters=(), dtype="bfloat16", full_config=True) -> ModelSpec:
    """A resolved ModelSpec for `cfg` (+ an optional nested hybrid transform config)."""
    resolved = cfg.to_dict() if full_config else {k: getattr(cfg, k) for k in CONFIG_KEYS}
    resolved["_load_dtype"] = dtype
    transforms = []
    if hybrid is not None:
        hy = dict(hybrid)
        lin = dict(hy["linear_attention"])
        if lin.get("linear_head_dim") is None:
            lin["linear_head_dim"] = cfg.attention_head_dim
        hy["linear_attention"] = lin
        transforms.append(TransformSpec(TRANSFORM_TYPE, HYBRID_TRANSFORM_VERSION, hy))
    spec = ModelSpec(format_version=2,
                     base=BaseSpec(library="diffusers", class_name="MiniMaxH3Transformer3DModel",
                                   source=source, subfolder="transformer", revision=None,
                                   resolved_config=resolved),
                     transforms=transforms, adapters=list(adapters))
    return validate_spec(spec)


def resolve_model_spec(model_section: Dict[str, Any], loaded_config: Dict[str, Any]) -> ModelSpec:
    """Stage A1's resolution: YAML architecture section + loaded base config -> spec."""
    base_cfg = model_section["base"]
    ha = model_section["architecture"]["hybrid_attention"]
    lin = dict(ha["linear_attention"])
    if lin.get("linear_head_dim") is None:
        lin["linear_head_dim"] = int(loaded_config["attention_head_dim"])
    if isinstance(lin.get("short_conv"), dict):
        lin["short_conv"] = {"targets": list(lin["short_conv"]["targets"])}
    resolved = dict(loaded_config)
    resolved["_load_dtype"] = base_cfg.get("dtype", "bfloat16")
    spec = ModelSpec(
        format_version=2,
        base=BaseSpec(library=base_cfg.get("library", "diffusers"),
                      class_name=base_cfg.get("class_name", "MiniMaxH3Transformer3DModel"),
                      source=base_cfg["source"], subfolder=base_cfg.get("subfolder", "transformer"),
                      revision=base_cfg.get("revision"), resolved_config=resolved),
        transforms=[TransformSpec(TRANSFORM_TYPE, HYBRID_TRANSFORM_VERSION, dict(
            enable_softmax_gate=ha["enable_softmax_gate"], anchor_frames=ha["anchor_frames"],
            softmax_attention=dict(ha["softmax_attention"]), linear_attention=lin))])
    return validate_spec(spec)


def load_model_weights(model, weights: Dict[str, torch.Tensor], strict=True):
    params = dict(model.named_parameters())
    missing = [k for k in weights if k not in params]
    if missing and strict:
        raise RuntimeError(f"{len(missing)} weight keys have no parameter, e.g. {sorted(missing)[:4]}")
    n = 0
    with torch.no_grad():
        for name, value in weights.items():
            if name in params:
                p = params[name]
                p.copy_(value.to(dtype=p.dtype, device=p.device))
                n += 1
    return n


RELEASED_HYBRID = dict(
    enable_softmax_gate=True, anchor_frames="both",
    softmax_attention=dict(radius=1, chunk=5),
    linear_attention=dict(delta_rule="vdn_solve", linear_head_dim=None, bridge="alpha",
                          short_conv=dict(targets=["k", "v"]), enable_text_state=True,
                          a_fp32=True))
"""The released checkpoints' transform (configs/training/stage_a1_c1_vdn_anchor.yaml:9-24):
c1 window (chunk 5, radius 1), anchors `both`, vdn_solve, K/V short conv, text state."""

TINY_HYBRID = dict(
    enable_softmax_gate=True, anchor_frames="none",
    softmax_attention=dict(radius=0, chunk=2),
    linear_attention=dict(delta_rule="sana_scaled", linear_head_dim=None, bridge="alpha",
                          short_conv=dict(targets=[]), enable_text_state=False, a_fp32=True))
"""The tiny CPU configuration's transform: a 2-frame window (chunk 2, radius 0), chunk-64 delta rule
(one 8x8 frame), beta = sigmoid(linear)."""
