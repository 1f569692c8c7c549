"""Atomic v2 writes: validate, write `<path>.tmp`, os.replace (reference
src/checkpoints/writer.py:12-20)."""
import os

import torch

from vdn_minimax_h3_b200.checkpoints.schema import CheckpointArtifact, validate_payload
from vdn_minimax_h3_b200.models.model_spec import ModelSpec


def save_checkpoint(artifact: CheckpointArtifact, path: str) -> str:
    payload = validate_payload(artifact.to_payload(), where=path)
    if "model_spec" in payload:
        ModelSpec.from_dict(payload["model_spec"])
    tmp = path + ".tmp"
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    torch.save(payload, tmp)
    os.replace(tmp, path)
    return path
