"""Checkpoint v2: what an artifact contains, and nothing else.

Reference parity: src/checkpoints/schema.py:19-95 (the same payload keys and kinds, because
the file format is the interchange contract: `weights`, `train_state`, `optimizer_shard`;
name-keyed optimizer state; pre-v2 meta stamps refused).
"""
from dataclasses import dataclass, field
from typing import Any, Dict, Optional

CHECKPOINT_FORMAT_VERSION = 2
ARTIFACT_KINDS = ("weights", "train_state", "optimizer_shard")
REQUIRED = {
    "weights": ("checkpoint_format_version", "kind", "model_spec", "weights"),
    "train_state": ("checkpoint_format_version", "kind", "model_spec", "weights", "step",
                    "rng_state", "resolved_training_config"),
    "optimizer_shard": ("checkpoint_format_version", "kind", "optimizer"),
}


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

    def to_payload(self):
        if self.kind == "optimizer_shard":
            return {"checkpoint_format_version": CHECKPOINT_FORMAT_VERSION, "kind": self.kind,
                    "optimizer": self.optimizer, "metadata": self.metadata}
        payload = {"checkpoint_format_version": CHECKPOINT_FORMAT_VERSION, "kind": self.kind,
                   "model_spec": self.model_spec, "weights": self.weights, "metadata": self.metadata}
        if self.kind == "train_state":
            payload.update(optimizer=self.optimizer, step=self.step, rng_state=self.rng_state,
                           resolved_training_config=self.resolved_training_config)
        return payload


def validate_payload(payload, where="checkpoint"):
    version = payload.get("checkpoint_format_version")
    if version != CHECKPOINT_FORMAT_VERSION:
        raise UnsupportedCheckpointFormat(
            f"{where}: unsupported checkpoint format {version if version is not None else 'pre-v2'}; "
            f"this code reads format {CHECKPOINT_FORMAT_VERSION} only")
    kind = payload.get("kind")
    if kind not in ARTIFACT_KINDS:
        raise UnsupportedCheckpointFormat(f"{where}: unknown artifact kind {kind!r}")
    missing = [k for k in REQUIRED[kind] if payload.get(k) is None]
    if missing:
        raise UnsupportedCheckpointFormat(f"{where}: {kind} artifact is missing {missing}")
    legacy = [k for k in payload.get("weights") or {} if k.startswith("__")]
    if legacy:
        raise UnsupportedCheckpointFormat(f"{where}: weights carry pre-v2 meta stamps {legacy}")
    if (kind == "train_state" and payload.get("optimizer") is None
            and not payload.get("metadata", {}).get("optimizer_shards")):
        raise UnsupportedCheckpointFormat(f"{where}: train_state carries neither an inline "
                                          f"optimizer nor metadata.optimizer_shards")
    opt = payload.get("optimizer")
    if opt is not None:
        bad = [k for k in opt if not isinstance(k, str)]
        if bad:
            raise UnsupportedCheckpointFormat(f"{where}: optimizer state must be keyed by "
                                              f"parameter NAME (got e.g. {bad[0]!r})")
    return payload
