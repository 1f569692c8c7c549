"""ModelSpec: the checkpoint-bound statement of WHAT the model is (base reference,
structural transforms, adapters). Runtime choices never enter it.

Reference parity: src/models/model_spec.py:1-179 (same JSON layout, same validator rules:
every value resolved, runtime keys refused, registries shared with the config schema,
legacy flat transform configs mapped through key_mapping).
"""
import hashlib
import json
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

from vdn_minimax_h3_b200.checkpoints.key_mapping import (ANCHOR_FRAME_MODES, DELTA_RULE_VALUES,
                                                         SHORT_CONV_TARGETS, map_config)

SPEC_FORMAT_VERSION = 2
HYBRID_TRANSFORM_VERSION = 2
BRIDGE_VALUES = ("alpha", "none")
RUNTIME_KEYS = ("softmax_backend", "rmsnorm_backend", "fp8", "compile", "inference_kernels",
                "optimized_paths", "w_o_far_scale", "window_decomp", "warmup_steps")


def config_hash(resolved_config: Dict[str, Any]) -> str:
    blob = json.dumps(resolved_config, sort_keys=True, separators=(",", ":"), default=str)
    return hashlib.sha256(blob.encode()).hexdigest()


@dataclass
class BaseSpec:
    library: str
    class_name: str
    source: str
    subfolder: str
    revision: Optional[str]
    resolved_config: Dict[str, Any]
    config_hash: str = ""

    def __post_init__(self):
        want = config_hash(self.resolved_config)
        if not self.config_hash:
            self.config_hash = want
        elif self.config_hash != want:
            raise ValueError(f"base.config_hash {self.config_hash[:12]} does not match "
                             f"resolved_config ({want[:12]})")


@dataclass
class TransformSpec:
    type: str
    version: int
    config: Dict[str, Any]


@dataclass
class AdapterSpec:
    type: str
    version: int
    config: Dict[str, Any]


@dataclass
class ModelSpec:
    format_version: int
    base: BaseSpec
    transforms: List[TransformSpec] = field(default_factory=list)
    adapters: List[AdapterSpec] = field(default_factory=list)

    def to_dict(self):
        return asdict(self)

    @staticmethod
    def from_dict(payload):
        spec = ModelSpec(format_version=payload["format_version"],
                         base=BaseSpec(**payload["base"]),
                         transforms=[TransformSpec(**t) for t in payload.get("transforms", [])],
                         adapters=[AdapterSpec(**a) for a in payload.get("adapters", [])])
        validate_spec(spec)
        return spec


def _flat_keys(config):
    for k, v in config.items():
        yield k
        if isinstance(v, dict):
            yield from _flat_keys(v)


def _require_resolved(config, where):
    for k, v in config.items():
        if v is None:
            raise ValueError(f"{where}.{k} is unresolved (null); a ModelSpec stores the value "
                             f"the model was built with")
        if isinstance(v, dict):
            _require_resolved(v, f"{where}.{k}")


def _validate_hybrid(config):
    lin = config.get("linear_attention", {})
    soft = config.get("softmax_attention", {})
    if lin.get("delta_rule") not in DELTA_RULE_VALUES:
        raise ValueError(f"delta_rule {lin.get('delta_rule')!r} not in {DELTA_RULE_VALUES}")
    if lin.get("bridge") not in BRIDGE_VALUES:
        raise ValueError(f"bridge {lin.get('bridge')!r} not in {BRIDGE_VALUES}")
    sc = lin.get("short_conv")
    targets = sc.get("targets") if isinstance(sc, dict) else None
    if (not isinstance(targets, list) or len(set(targets)) != len(targets)
            or any(t not in SHORT_CONV_TARGETS for t in targets)):
        raise ValueError(f"short_conv must be {{'targets': subset of {SHORT_CONV_TARGETS}}}, "
                         f"got {sc!r}")
    if config.get("anchor_frames") not in ANCHOR_FRAME_MODES:
        raise ValueError(f"anchor_frames {config.get('anchor_frames')!r} not in {ANCHOR_FRAME_MODES}")
    if not isinstance(lin.get("linear_head_dim"), int):
        raise ValueError(f"linear_head_dim must be a resolved int, got {lin.get('linear_head_dim')!r}")
    if not isinstance(soft.get("radius"), int):
        raise ValueError(f"softmax_attention.radius must be a resolved int, got {soft.get('radius')!r}")
    if not isinstance(config.get("enable_softmax_gate"), bool):
        raise ValueError("enable_softmax_gate must be a resolved bool")


def validate_spec(spec: ModelSpec):
    if spec.format_version != SPEC_FORMAT_VERSION:
        raise ValueError(f"spec format_version {spec.format_version} != {SPEC_FORMAT_VERSION}")
    for t in spec.transforms:
        _require_resolved(t.config, f"transforms[{t.type}]")
        leaked = sorted(set(_flat_keys(t.config)) & set(RUNTIME_KEYS))
        if leaked:
            raise ValueError(f"transforms[{t.type}] carries runtime keys {leaked}")
        if t.type == "hybrid_attention":
            if t.version != HYBRID_TRANSFORM_VERSION:
                raise ValueError(f"hybrid_attention transform version {t.version}; this code "
                                 f"reads version {HYBRID_TRANSFORM_VERSION}")
            _validate_hybrid(t.config)
    for a in spec.adapters:
        _require_resolved(a.config, f"adapters[{a.type}]")
    return spec


def hybrid_transform_spec(legacy_or_nested):
    """TransformSpec from either the flat pre-v2 kwargs or the nested v2 layout."""
    if "softmax_attention" in legacy_or_nested:
        nested = dict(legacy_or_nested)
    else:
        flat = map_config(dict(legacy_or_nested))
        nested = dict(enable_softmax_gate=flat.pop("enable_softmax_gate", True),
                      anchor_frames=flat.pop("anchor_frames", "none"),
                      softmax_attention=dict(radius=flat.pop("radius"), chunk=flat.pop("chunk", 0)),
                      linear_attention=flat)
    return TransformSpec("hybrid_attention", HYBRID_TRANSFORM_VERSION, nested)
