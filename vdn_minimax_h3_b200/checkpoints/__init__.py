"""Checkpoint v2 (schema, loader, writer, exploded directory, key mapping).

Names are resolved lazily so that `checkpoints.key_mapping` (used by the ModelSpec) can be
imported without pulling in the loaders, which themselves import the ModelSpec."""
_EXPORTS = {
    "export_checkpoint_dir": "export_dir", "load_checkpoint_dir": "export_dir",
    "checkpoint_head_sha256": "loader", "load_checkpoint": "loader",
    "CheckpointArtifact": "schema", "UnsupportedCheckpointFormat": "schema",
    "validate_payload": "schema", "save_checkpoint": "writer",
}


def __getattr__(name):
    if name in _EXPORTS:
        import importlib
        mod = importlib.import_module(f"vdn_minimax_h3_b200.checkpoints.{_EXPORTS[name]}")
        return getattr(mod, name)
    raise AttributeError(name)
