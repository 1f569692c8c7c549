"""Reading checkpoints: a v2 `.pt` file or an exploded directory becomes a
CheckpointArtifact; anything else raises UnsupportedCheckpointFormat (there is no shim for
older formats). Behaviour parity: src/checkpoints/loader.py:13-61.

`checkpoint_head_sha256` is the identity stamp a render record carries: cheap to compute on
a 60 GB file (it reads at most 1 MiB of tensor data per file) yet it changes whenever the
weights it samples change.
"""
import dataclasses
import hashlib
import os
import struct

import torch

from vdn_minimax_h3_b200.checkpoints.export_dir import is_checkpoint_dir, load_checkpoint_dir
from vdn_minimax_h3_b200.checkpoints.schema import (CheckpointArtifact, UnsupportedCheckpointFormat,
                                                    validate_payload)
from vdn_minimax_h3_b200.models.model_spec import ModelSpec

_SAMPLE = 1 << 20


def _file_digest(path: str) -> str:
    """sha256 of a file's leading MiB; for safetensors, of its tensor table (the JSON
    header: names, dtypes, shapes, offsets) plus the leading MiB of the data after it."""
    h = hashlib.sha256()
    with open(path, "rb") as f:
        if path.endswith(".safetensors"):
            (n,) = struct.unpack("<Q", f.read(8))
            h.update(f.read(n))
        h.update(f.read(_SAMPLE))
    return h.hexdigest()


def checkpoint_head_sha256(path: str) -> str:
    """Identity stamp of a `.pt` file or an exploded directory (every member, by its
    relative path, in sorted order)."""
    if not is_checkpoint_dir(path):
        return _file_digest(path)
    lines = []
    for root, _, files in os.walk(path):
        for name in files:
            full = os.path.join(root, name)
            lines.append(f"{os.path.relpath(full, path)}\0{_file_digest(full)}\n")
    return hashlib.sha256("".join(sorted(lines)).encode()).hexdigest()


def _read_payload(path: str, mmap: bool) -> dict:
    try:
        payload = torch.load(path, map_location="cpu", weights_only=True, mmap=mmap)
    except Exception as exc:  # noqa: BLE001 - any unreadable file is the same refusal
        raise UnsupportedCheckpointFormat(
            f"{path}: cannot be read as a checkpoint ({type(exc).__name__}: {exc})") from exc
    if not isinstance(payload, dict):
        raise UnsupportedCheckpointFormat(f"{path}: the payload is a {type(payload).__name__}, "
                                          f"not a dict")
    return validate_payload(payload, where=path)


def load_checkpoint(path: str, mmap: bool = True) -> CheckpointArtifact:
    if is_checkpoint_dir(path):
        return load_checkpoint_dir(path)
    payload = _read_payload(path, mmap)
    if payload.get("model_spec") is not None:
        ModelSpec.from_dict(payload["model_spec"])          # refuses an invalid spec
    values = {f.name: payload.get(f.name) for f in dataclasses.fields(CheckpointArtifact)}
    values["metadata"] = values["metadata"] or {}
    return CheckpointArtifact(**values)
