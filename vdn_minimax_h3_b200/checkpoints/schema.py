"""Checkpoint format v2: the artifact kinds, which fields each kind stores, and the checks
a payload must pass before it is written or after it is read.

The kinds and field names are the reference's file format (src/checkpoints/schema.py:
19-95), kept so checkpoints move between the two: `weights` (model_spec + weights),
`train_state` (those + optimizer, step, rng_state, resolved_training_config) and
`optimizer_shard` (one rank's ZeRO-1 moments). Optimizer state is keyed by parameter name.
Here each kind is a row of one table, and each rule is a small function over the payload.
"""
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Tuple

CHECKPOINT_FORMAT_VERSION = 2

# kind -> (fields written, fields that must be present and non-null)
_KINDS: Dict[str, Tuple[Tuple[str, ...], Tuple[str, ...]]] = {
    "weights": (("model_spec", "weights", "metadata"), ("model_spec", "weights")),
    "train_state": (("model_spec", "weights", "metadata", "optimizer", "step", "rng_state",
                     "resolved_training_config"),
                    ("model_spec", "weights", "step", "rng_state", "resolved_training_config")),
    "optimizer_shard": (("optimizer", "metadata"), ("optimizer",)),
}
ARTIFACT_KINDS = tuple(_KINDS)
REQUIRED = {k: ("checkpoint_format_version", "kind") + req for k, (_, req) in _KINDS.items()}


class UnsupportedCheckpointFormat(RuntimeError):
    pass


@dataclass
class CheckpointArtifact:
    kind: str
    model_spec: Optional[Dict[str, Any]]
    weights: Optional[Dict[str, Any]]
    optimizer: Optional[Dict[str, Any]] = None
    step: Optional[int] = None
    rng_state: Optional[Dict[str, Any]] = None
    resolved_training_config: Optional[Dict[str, Any]] = None
    metadata: Dict[str, Any] = field(default_factory=dict)

    def to_payload(self) -> Dict[str, Any]:
        if self.kind not in _KINDS:
            raise UnsupportedCheckpointFormat(f"unknown artifact kind {self.kind!r}")
        stored, _ = _KINDS[self.kind]
        payload = {"checkpoint_format_version": CHECKPOINT_FORMAT_VERSION, "kind": self.kind}
        payload.update((name, getattr(self, name)) for name in stored)
        return payload


# Each rule: payload -> problem text, or None. They run in order after the version and
# kind checks; the first problem is raised.
def _missing_fields(p):
    gone = [k for k in REQUIRED[p["kind"]] if p.get(k) is None]
    return f"{p['kind']} artifact is missing {gone}" if gone else None


def _meta_stamps_in_weights(p):
    stamps = [k for k in (p.get("weights") or {}) if str(k).startswith("__")]
    return f"weights carry pre-v2 meta stamps {stamps}" if stamps else None


def _optimizer_location(p):
    if p["kind"] != "train_state" or p.get("optimizer") is not None:
        return None
    if (p.get("metadata") or {}).get("optimizer_shards"):
        return None
    return "train_state carries neither an inline optimizer nor metadata.optimizer_shards"


def _optimizer_keys(p):
    for key in p.get("optimizer") or {}:
        if not isinstance(key, str):
            return f"optimizer state must be keyed by parameter NAME (found key {key!r})"
    return None


_RULES: List[Callable[[Dict[str, Any]], Optional[str]]] = [
    _missing_fields, _meta_stamps_in_weights, _optimizer_location, _optimizer_keys]


def validate_payload(payload: Dict[str, Any], where: str = "checkpoint") -> Dict[str, Any]:
    version = payload.get("checkpoint_format_version")
    if version != CHECKPOINT_FORMAT_VERSION:
        shown = "pre-v2" if version is None else version
        raise UnsupportedCheckpointFormat(
            f"{where}: checkpoint format {shown} is not readable; format "
            f"{CHECKPOINT_FORMAT_VERSION} is the only one this code reads")
    if payload.get("kind") not in _KINDS:
        raise UnsupportedCheckpointFormat(f"{where}: unknown artifact kind {payload.get('kind')!r}")
    for rule in _RULES:
        problem = rule(payload)
        if problem:
            raise UnsupportedCheckpointFormat(f"{where}: {problem}")
    return payload
