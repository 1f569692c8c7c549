"""The one reader: a v2 `.pt` or the exploded directory -> CheckpointArtifact; anything
else is refused (reference src/checkpoints/loader.py:13-61), plus the identity stamp of a
render record (sha256 over the first MiB of the file, or of each directory member's data)."""
import hashlib
import os
import struct

import torch

from vdn_minimax_h3_b200.checkpoints.export_dir import is_checkpoint_dir, load_checkpoint_dir
from vdn_minimax_h3_b200.checkpoints.schema import (CheckpointArtifact, UnsupportedCheckpointFormat,
                                                    validate_payload)
from vdn_minimax_h3_b200.models.model_spec import ModelSpec


def checkpoint_head_sha256(path):
    digest = hashlib.sha256()
    if not is_checkpoint_dir(path):
        with open(path, "rb") as f:
            digest.update(f.read(1 << 20))
        return digest.hexdigest()
    for root, _, files in sorted(os.walk(path)):
        for name in sorted(files):
            with open(os.path.join(root, name), "rb") as f:
                if name.endswith(".safetensors"):
                    n = struct.unpack("<Q", f.read(8))[0]
                    f.seek(8 + n)
                digest.update(name.encode())
                digest.update(f.read(1 << 20))
    return digest.hexdigest()


def load_checkpoint(path, mmap=True):
    if is_checkpoint_dir(path):
        return load_checkpoint_dir(path)
    try:
        payload = torch.load(path, map_location="cpu", weights_only=True, mmap=mmap)
    except Exception as exc:  # noqa: BLE001
        raise UnsupportedCheckpointFormat(f"{path}: not a readable checkpoint "
                                          f"({type(exc).__name__}: {exc})") from exc
    if not isinstance(payload, dict):
        raise UnsupportedCheckpointFormat(f"{path}: expected a dict payload")
    validate_payload(payload, where=path)
    if payload.get("model_spec") is not None:
        ModelSpec.from_dict(payload["model_spec"])
    return CheckpointArtifact(kind=payload["kind"], model_spec=payload.get("model_spec"),
                              weights=payload.get("weights"), optimizer=payload.get("optimizer"),
                              step=payload.get("step"), rng_state=payload.get("rng_state"),
                              resolved_training_config=payload.get("resolved_training_config"),
                              metadata=payload.get("metadata", {}))
