"""Command-line entry of the four training stages.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m vdn_minimax_h3_b200.training.train \
        b --config configs/training/stage_b_c1_vdn_anchor.yaml data.index_file=/path/index.jsonl \
        [more.dotlist=overrides]

The first argument picks the stage (a1 | a2 | b | dmd); the rest is the layered config of
vdn_minimax_h3_b200.config (YAML, then `key=value` overrides; `--print-config` /
`--validate-only` stop after the config). One process per GPU under torchrun (NCCL;
RANK / LOCAL_RANK / WORLD_SIZE / MASTER_* from the environment), or one CPU process on gloo
when CUDA is absent. Returns the last completed step.

| stage | config file | what trains |
|---|---|---|
| a1 | configs/training/stage_a1_c1_vdn_anchor.yaml | the hybrid branch, per layer against the dense teacher (DDP + ZeRO-1) |
| a2 | configs/training/stage_a2_c1_vdn_anchor.yaml | the hybrid branch end to end against the teacher velocity (FSDP2) |
| b | configs/training/stage_b_c1_vdn_anchor.yaml | the branch + the `default` LoRA, teacher and data losses (FSDP2) |
| dmd | configs/training/stage_dmd_vdn.yaml | DMD2 few-step generator, real / fake score (FSDP2) |

Reference parity: the per-stage launchers scripts/training/stage_{a1,a2,b,dmd_vdn}.sh and
the entry scripts src/training/train_stage_{a1,a2,b,dmd}.py (one module per stage there,
one module with a stage argument here; the configs and their keys are the same).
"""
import sys

import torch.distributed as dist

from vdn_minimax_h3_b200.config import load_config
from vdn_minimax_h3_b200.config.schemas import (StageA1Config, StageA2Config, StageBConfig,
                                                StageDMDConfig, validate_enums, validate_stage_dmd)

STAGES = {
    "a1": (StageA1Config, (validate_enums,), "run_stage_a1"),
    "a2": (StageA2Config, (), "run_stage_a2"),
    "b": (StageBConfig, (), "run_stage_b"),
    "dmd": (StageDMDConfig, (validate_stage_dmd,), "run_stage_dmd"),
}


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] not in STAGES:
        raise SystemExit(f"usage: train {{{'|'.join(STAGES)}}} --config FILE [key=value ...]")
    stage, rest = argv[0], argv[1:]
    schema, validators, fn_name = STAGES[stage]
    cfg = load_config(schema, rest, validators)
    from vdn_minimax_h3_b200.training import trainers
    try:
        return getattr(trainers, fn_name)(cfg)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
    sys.exit(0)
