"""ModelSpec: what a checkpoint's model IS -- the base it starts from, the structural
transforms applied to it and the adapters it carries. How a run executes it (kernels, fp8,
parallelism) is runtime configuration and is refused here, so a checkpoint never pins a
kernel choice.

The JSON layout (format_version 2: `base`, `transforms[]`, `adapters[]` with
`{type, version, config}` entries) and the base-config hash (sha256 over the canonical
JSON rendering) are the reference's on-disk format (src/models/model_spec.py:18-95); the
validation here is table driven: every problem of a spec is collected and reported in one
error, rather than stopping at the first.
"""
import hashlib
import json
from dataclasses import asdict, dataclass, field
from typing import Any, Callable, Dict, Iterator, List, NamedTuple, Optional, Tuple

from vdn_minimax_h3_b200.checkpoints.key_mapping import (ANCHOR_FRAME_MODES, DELTA_RULE_VALUES,
                                                         SHORT_CONV_TARGETS, map_config)

SPEC_FORMAT_VERSION = 2
HYBRID_TRANSFORM_VERSION = 2
BRIDGE_VALUES = ("alpha", "none")
# Execution knobs, present and retired: a transform config naming any of them is refused,
# wherever in the nesting the key appears.
RUNTIME_KEYS = frozenset(("softmax_backend", "rmsnorm_backend", "fp8", "compile",
                          "inference_kernels", "optimized_paths", "w_o_far_scale",
                          "window_decomp", "warmup_steps"))


def _canonical(obj: Any) -> str:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"), default=str)


def config_hash(resolved_config: Dict[str, Any]) -> str:
    """Hex sha256 of the canonical JSON text: independent of key order."""
    return hashlib.sha256(_canonical(resolved_config).encode()).hexdigest()


class SpecError(ValueError):
    """A ModelSpec that cannot be stored or loaded; lists every problem found."""

    def __init__(self, problems: List[str]):
        self.problems = list(problems)
        super().__init__("invalid ModelSpec:\n  - " + "\n  - ".join(self.problems))


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
        digest = config_hash(self.resolved_config)
        if self.config_hash and self.config_hash != digest:
            raise SpecError([f"base.config_hash {self.config_hash[:12]}... was not computed "
                             f"from base.resolved_config (hash {digest[:12]}...)"])
        self.config_hash = digest


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

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)

    @staticmethod
    def from_dict(payload: Dict[str, Any]) -> "ModelSpec":
        entries = lambda kind, cls: [cls(**e) for e in payload.get(kind, [])]  # noqa: E731
        return validate_spec(ModelSpec(payload["format_version"], BaseSpec(**payload["base"]),
                                       entries("transforms", TransformSpec),
                                       entries("adapters", AdapterSpec)))


def _walk(config: Dict[str, Any], prefix: str) -> Iterator[Tuple[str, str, Any]]:
    """(dotted path, key, value) for every entry of a nested config, parents first."""
    for key, value in config.items():
        path = f"{prefix}.{key}"
        yield path, key, value
        if isinstance(value, dict):
            yield from _walk(value, path)


def _storage_problems(config: Dict[str, Any], where: str, runtime_keys=RUNTIME_KEYS) -> List[str]:
    out = []
    for path, key, value in _walk(config, where):
        if value is None:
            out.append(f"{path} is null: a spec stores the value the model was built with")
        if key in runtime_keys:
            out.append(f"{path} is a runtime setting and never enters a ModelSpec")
    return out


class _Rule(NamedTuple):
    path: Tuple[str, ...]                 # key path inside the hybrid transform's config
    ok: Callable[[Any], bool]
    expected: str


def _targets_ok(short_conv: Any) -> bool:
    if not isinstance(short_conv, dict) or not isinstance(short_conv.get("targets"), list):
        return False
    targets = short_conv["targets"]
    return len(set(targets)) == len(targets) and set(targets) <= set(SHORT_CONV_TARGETS)


_HYBRID_RULES = (
    _Rule(("linear_attention", "delta_rule"), lambda v: v in DELTA_RULE_VALUES,
          f"one of {DELTA_RULE_VALUES}"),
    _Rule(("linear_attention", "bridge"), lambda v: v in BRIDGE_VALUES, f"one of {BRIDGE_VALUES}"),
    _Rule(("linear_attention", "short_conv"), _targets_ok,
          f"{{'targets': [distinct entries of {SHORT_CONV_TARGETS}]}}"),
    _Rule(("linear_attention", "linear_head_dim"), lambda v: type(v) is int, "an int"),
    _Rule(("softmax_attention", "radius"), lambda v: type(v) is int, "an int"),
    _Rule(("anchor_frames",), lambda v: v in ANCHOR_FRAME_MODES, f"one of {ANCHOR_FRAME_MODES}"),
    _Rule(("enable_softmax_gate",), lambda v: type(v) is bool, "a bool"),
)
_MISSING = object()


def _lookup(config: Dict[str, Any], path: Tuple[str, ...]) -> Any:
    node: Any = config
    for key in path:
        node = node.get(key, _MISSING) if isinstance(node, dict) else _MISSING
    return node


def _hybrid_problems(t: TransformSpec) -> List[str]:
    if t.version != HYBRID_TRANSFORM_VERSION:
        return [f"hybrid_attention transform version {t.version} is not readable here "
                f"(this code reads version {HYBRID_TRANSFORM_VERSION})"]
    out = []
    for rule in _HYBRID_RULES:
        value = _lookup(t.config, rule.path)
        if value is _MISSING or not rule.ok(value):
            shown = "missing" if value is _MISSING else repr(value)
            out.append(f"hybrid_attention {'.'.join(rule.path)} = {shown}; expected {rule.expected}")
    return out


def validate_spec(spec: ModelSpec) -> ModelSpec:
    """Returns the spec when it is storable; raises SpecError listing every problem."""
    problems = []
    if spec.format_version != SPEC_FORMAT_VERSION:
        problems.append(f"format_version {spec.format_version} (this code reads {SPEC_FORMAT_VERSION})")
    for t in spec.transforms:
        problems += _storage_problems(t.config, f"transforms[{t.type}]")
        if t.type == "hybrid_attention":
            problems += _hybrid_problems(t)
    for a in spec.adapters:
        problems += _storage_problems(a.config, f"adapters[{a.type}]", runtime_keys=())
    if problems:
        raise SpecError(problems)
    return spec


# Flat pre-v2 kwargs that belong outside `linear_attention` in the nested v2 layout:
# (flat key, nested destination, default when absent).
_FLAT_TO_NESTED = (("enable_softmax_gate", ("enable_softmax_gate",), True),
                   ("anchor_frames", ("anchor_frames",), "none"),
                   ("radius", ("softmax_attention", "radius"), _MISSING),
                   ("chunk", ("softmax_attention", "chunk"), 0))


def hybrid_transform_spec(kwargs: Dict[str, Any]) -> TransformSpec:
    """The v2 TransformSpec of the hybrid attention from either the nested v2 config or the
    flat pre-v2 conversion kwargs (renamed through key_mapping.map_config); whatever the
    flat form does not place elsewhere is the `linear_attention` block."""
    if "softmax_attention" in kwargs:
        return TransformSpec("hybrid_attention", HYBRID_TRANSFORM_VERSION, dict(kwargs))
    rest = map_config(dict(kwargs))
    nested: Dict[str, Any] = {"softmax_attention": {}}
    for flat_key, dest, default in _FLAT_TO_NESTED:
        value = rest.pop(flat_key, default)
        if value is _MISSING:
            raise KeyError(f"pre-v2 hybrid kwargs lack {flat_key!r}")
        (nested if len(dest) == 1 else nested[dest[0]])[dest[-1]] = value
    nested["linear_attention"] = rest
    return TransformSpec("hybrid_attention", HYBRID_TRANSFORM_VERSION, nested)
