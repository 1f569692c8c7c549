from vdn_minimax_h3_b200.checkpoints.export_dir import export_checkpoint_dir, load_checkpoint_dir  # noqa: F401
from vdn_minimax_h3_b200.checkpoints.loader import checkpoint_head_sha256, load_checkpoint  # noqa: F401
from vdn_minimax_h3_b200.checkpoints.schema import (CheckpointArtifact,  # noqa: F401
                                                    UnsupportedCheckpointFormat, validate_payload)
from vdn_minimax_h3_b200.checkpoints.writer import save_checkpoint  # noqa: F401
