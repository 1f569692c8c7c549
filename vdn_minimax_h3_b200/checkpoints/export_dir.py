"""The exploded checkpoint directory: a `weights` artifact with its JSON and its tensors
in separate, individually readable files.

    OUT_DIR/
      model_spec.json, metadata.json
      linear_branch/{config.json, model.safetensors}
      adapters/<name>/{adapter_spec.json, adapter_model.safetensors}

The layout and file names are the release format of existing checkpoints
(src/checkpoints/export_dir.py:1-25), so both implementations read each other's exports.
Writing builds the whole tree in a private temporary directory beside OUT_DIR and renames
it into place, so a reader never sees a half-written export; a failed export leaves
nothing behind.

    python -m vdn_minimax_h3_b200.checkpoints.export_dir IN.pt OUT_DIR [--dtype bfloat16|float32|keep]
"""
import argparse
import json
import os
import re
import shutil
import tempfile
from typing import Callable, Dict, List, Tuple

import torch

from vdn_minimax_h3_b200.checkpoints.schema import (CHECKPOINT_FORMAT_VERSION, CheckpointArtifact,
                                                    UnsupportedCheckpointFormat)
from vdn_minimax_h3_b200.models.model_spec import ModelSpec

SPEC_FILE, META_FILE = "model_spec.json", "metadata.json"
BRANCH_DIR, ADAPTERS_DIR = "linear_branch", "adapters"
BRANCH_CONFIG, BRANCH_TENSORS = "config.json", "model.safetensors"
ADAPTER_SPEC, ADAPTER_TENSORS = "adapter_spec.json", "adapter_model.safetensors"
# peft tensor names: `<module>.lora_A.<adapter>.weight` / `lora_B`
_ADAPTER_OF = re.compile(r"\.lora_[AB]\.(?P<adapter>[^.]+)\.")


def adapter_name_of(key: str):
    """The adapter a peft LoRA tensor belongs to; None for every other tensor."""
    hit = _ADAPTER_OF.search(key)
    return hit.group("adapter") if hit else None


def split_weights(weights):
    """(branch tensors, {adapter name: its tensors})."""
    groups: Dict[str, Dict[str, torch.Tensor]] = {}
    for key, tensor in weights.items():
        groups.setdefault(adapter_name_of(key) or "", {})[key] = tensor
    branch = groups.pop("", {})
    return branch, groups


def match_adapter_specs(spec: dict, names: List[str]) -> Dict[str, dict]:
    """Pairs each adapter present in the tensors with its ModelSpec entry: an entry whose
    config names the adapter; else peft's unnamed first entry for `default`; else the entry
    at the adapter's position."""
    entries = spec.get("adapters", [])
    by_name = {e["config"]["name"]: e for e in entries if "name" in e["config"]}
    out = {}
    for pos, name in enumerate(names):
        if name in by_name:
            out[name] = by_name[name]
        elif name == "default" and entries and "name" not in entries[0]["config"]:
            out[name] = entries[0]
        elif pos < len(entries):
            out[name] = entries[pos]
        else:
            raise UnsupportedCheckpointFormat(f"adapter {name!r} has tensors but the spec "
                                              f"has no entry for it")
    return out


def _json_writer(obj) -> Callable[[str], None]:
    def write(path):
        with open(path, "w") as f:
            f.write(json.dumps(obj, indent=2, sort_keys=True) + "\n")
    return write


def _tensor_writer(tensors, cast) -> Callable[[str], None]:
    def write(path):
        from safetensors.torch import save_file
        ready = {k: (t.to(cast) if cast is not None and t.is_floating_point() else t).contiguous()
                 for k, t in tensors.items()}
        save_file(ready, path)
    return write


def _export_plan(artifact: CheckpointArtifact, dtype: str) -> List[Tuple[str, Callable]]:
    """(path relative to OUT_DIR, writer) for every file of the export."""
    spec = artifact.model_spec
    cast = None if dtype == "keep" else getattr(torch, dtype)
    branch, adapters = split_weights(artifact.weights)
    transforms = spec.get("transforms", [])
    plan = [(SPEC_FILE, _json_writer(spec)),
            (META_FILE, _json_writer({"kind": artifact.kind, "weights_dtype": dtype,
                                      "checkpoint_format_version": CHECKPOINT_FORMAT_VERSION,
                                      "metadata": artifact.metadata})),
            (os.path.join(BRANCH_DIR, BRANCH_CONFIG), _json_writer(transforms[0] if transforms else {})),
            (os.path.join(BRANCH_DIR, BRANCH_TENSORS), _tensor_writer(branch, cast))]
    specs = match_adapter_specs(spec, list(adapters))
    for name, tensors in adapters.items():
        plan.append((os.path.join(ADAPTERS_DIR, name, ADAPTER_SPEC), _json_writer(specs[name])))
        plan.append((os.path.join(ADAPTERS_DIR, name, ADAPTER_TENSORS), _tensor_writer(tensors, cast)))
    return plan


def export_checkpoint_dir(artifact: CheckpointArtifact, out_dir, dtype="bfloat16"):
    if artifact.kind != "weights":
        raise UnsupportedCheckpointFormat(f"a {artifact.kind!r} artifact is not exportable; "
                                          f"only `weights` artifacts are")
    ModelSpec.from_dict(artifact.model_spec)
    out_dir = out_dir.rstrip("/")
    if os.path.exists(out_dir):
        raise FileExistsError(f"{out_dir} already exists; exports never overwrite")
    plan = _export_plan(artifact, dtype)
    parent = os.path.dirname(os.path.abspath(out_dir))
    os.makedirs(parent, exist_ok=True)
    staging = tempfile.mkdtemp(prefix=f".{os.path.basename(out_dir)}.", suffix=".partial", dir=parent)
    try:
        for rel, write in plan:
            os.makedirs(os.path.dirname(os.path.join(staging, rel)), exist_ok=True)
            write(os.path.join(staging, rel))
        os.replace(staging, out_dir)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise
    return out_dir


def is_checkpoint_dir(path):
    return os.path.isdir(path) and os.path.isfile(os.path.join(path, SPEC_FILE))


def load_checkpoint_dir(path):
    from safetensors.torch import load_file

    def read_json(rel):
        with open(os.path.join(path, rel)) as f:
            return json.load(f)

    spec, meta = read_json(SPEC_FILE), read_json(META_FILE)
    if (meta.get("kind"), meta.get("checkpoint_format_version")) != ("weights", CHECKPOINT_FORMAT_VERSION):
        raise UnsupportedCheckpointFormat(f"{path}: metadata does not describe a format-"
                                          f"{CHECKPOINT_FORMAT_VERSION} `weights` export")
    ModelSpec.from_dict(spec)
    weights = load_file(os.path.join(path, BRANCH_DIR, BRANCH_TENSORS))
    adapters_root = os.path.join(path, ADAPTERS_DIR)
    names = sorted(os.listdir(adapters_root)) if os.path.isdir(adapters_root) else []
    for name in names:
        weights.update(load_file(os.path.join(adapters_root, name, ADAPTER_TENSORS)))
    return CheckpointArtifact(kind="weights", model_spec=spec, weights=weights,
                              metadata=meta.get("metadata", {}))


def main(argv=None):
    from vdn_minimax_h3_b200.checkpoints.loader import load_checkpoint
    p = argparse.ArgumentParser(description="write a v2 `weights` checkpoint as an exploded directory")
    p.add_argument("checkpoint")
    p.add_argument("out_dir")
    p.add_argument("--dtype", default="bfloat16", choices=("bfloat16", "float32", "keep"))
    a = p.parse_args(argv)
    art = load_checkpoint(a.checkpoint)
    out = export_checkpoint_dir(art, a.out_dir, dtype=a.dtype)
    branch, adapters = split_weights(art.weights)
    sizes = {"linear_branch": len(branch), **{f"adapters/{n}": len(t) for n, t in adapters.items()}}
    print(json.dumps({"exported": out, "dtype": a.dtype, "tensors": sizes}))


if __name__ == "__main__":
    main()
