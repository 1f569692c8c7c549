"""The exploded checkpoint directory: one `weights` artifact, config and tensors apart.

    OUT_DIR/
      model_spec.json, metadata.json
      linear_branch/{config.json, model.safetensors}
      adapters/<name>/{adapter_spec.json, adapter_model.safetensors}

Reference parity: src/checkpoints/export_dir.py:1-167 (the same layout and file names: it
is the release format existing checkpoints ship in). Written to `<out>.tmp` and renamed.

    python -m vdn_minimax_h3_b200.checkpoints.export_dir IN.pt OUT_DIR [--dtype bfloat16|float32|keep]
"""
import argparse
import json
import os
import re

import torch

from vdn_minimax_h3_b200.checkpoints.schema import CheckpointArtifact, UnsupportedCheckpointFormat
from vdn_minimax_h3_b200.models.model_spec import ModelSpec

SPEC_FILE, META_FILE = "model_spec.json", "metadata.json"
BRANCH_DIR, ADAPTERS_DIR = "linear_branch", "adapters"
_LORA_KEY = re.compile(r"\.lora_[AB]\.([^.]+)\.")


def adapter_name_of(key):
    m = _LORA_KEY.search(key)
    return m.group(1) if m else None


def split_weights(weights):
    branch, adapters = {}, {}
    for key, t in weights.items():
        name = adapter_name_of(key)
        if name is None:
            branch[key] = t
        else:
            adapters.setdefault(name, {})[key] = t
    return branch, adapters


def _adapter_entry(spec, name, index):
    entries = spec.get("adapters", [])
    for e in entries:
        if e["config"].get("name") == name:
            return e
    if name == "default" and entries and "name" not in entries[0]["config"]:
        return entries[0]
    if index < len(entries):
        return entries[index]
    raise UnsupportedCheckpointFormat(f"adapter {name!r} has tensors but no spec entry")


def _dump(obj, path):
    with open(path, "w") as f:
        json.dump(obj, f, indent=2, sort_keys=True)
        f.write("\n")


def export_checkpoint_dir(artifact: CheckpointArtifact, out_dir, dtype="bfloat16"):
    from safetensors.torch import save_file
    if artifact.kind != "weights":
        raise UnsupportedCheckpointFormat(f"only `weights` artifacts are exported, got {artifact.kind!r}")
    ModelSpec.from_dict(artifact.model_spec)
    cast = None if dtype == "keep" else getattr(torch, dtype)

    def prepared(ts):
        return {k: (t.to(cast) if cast is not None and t.is_floating_point() else t).contiguous()
                for k, t in ts.items()}

    branch, adapters = split_weights(artifact.weights)
    tmp = out_dir.rstrip("/") + ".tmp"
    if os.path.exists(tmp):
        raise FileExistsError(f"{tmp} exists; a previous export did not finish")
    os.makedirs(os.path.join(tmp, BRANCH_DIR))
    _dump(artifact.model_spec, os.path.join(tmp, SPEC_FILE))
    _dump({"kind": artifact.kind, "checkpoint_format_version": 2, "weights_dtype": dtype,
           "metadata": artifact.metadata}, os.path.join(tmp, META_FILE))
    transforms = artifact.model_spec.get("transforms", [])
    _dump(transforms[0] if transforms else {}, os.path.join(tmp, BRANCH_DIR, "config.json"))
    save_file(prepared(branch), os.path.join(tmp, BRANCH_DIR, "model.safetensors"))
    for i, (name, ts) in enumerate(adapters.items()):
        adir = os.path.join(tmp, ADAPTERS_DIR, name)
        os.makedirs(adir)
        _dump(_adapter_entry(artifact.model_spec, name, i), os.path.join(adir, "adapter_spec.json"))
        save_file(prepared(ts), os.path.join(adir, "adapter_model.safetensors"))
    if os.path.exists(out_dir):
        raise FileExistsError(f"{out_dir} exists; remove it first")
    os.replace(tmp, out_dir)
    return out_dir


def is_checkpoint_dir(path):
    return os.path.isdir(path) and os.path.isfile(os.path.join(path, SPEC_FILE))


def load_checkpoint_dir(path):
    from safetensors.torch import load_file
    with open(os.path.join(path, SPEC_FILE)) as f:
        spec = json.load(f)
    with open(os.path.join(path, META_FILE)) as f:
        meta = json.load(f)
    if meta.get("checkpoint_format_version") != 2 or meta.get("kind") != "weights":
        raise UnsupportedCheckpointFormat(f"{path}: not an exploded `weights` artifact")
    ModelSpec.from_dict(spec)
    weights = load_file(os.path.join(path, BRANCH_DIR, "model.safetensors"))
    root = os.path.join(path, ADAPTERS_DIR)
    if os.path.isdir(root):
        for name in sorted(os.listdir(root)):
            weights.update(load_file(os.path.join(root, name, "adapter_model.safetensors")))
    return CheckpointArtifact(kind="weights", model_spec=spec, weights=weights,
                              metadata=meta.get("metadata", {}))


def main(argv=None):
    from vdn_minimax_h3_b200.checkpoints.loader import load_checkpoint
    p = argparse.ArgumentParser(description="export a v2 weights artifact as a directory")
    p.add_argument("checkpoint")
    p.add_argument("out_dir")
    p.add_argument("--dtype", default="bfloat16", choices=("bfloat16", "float32", "keep"))
    a = p.parse_args(argv)
    art = load_checkpoint(a.checkpoint)
    out = export_checkpoint_dir(art, a.out_dir, dtype=a.dtype)
    branch, adapters = split_weights(art.weights)
    print(f"wrote {out}: {len(branch)} branch tensors, "
          + ", ".join(f"adapter {n}: {len(t)} tensors" for n, t in adapters.items()))


if __name__ == "__main__":
    main()
