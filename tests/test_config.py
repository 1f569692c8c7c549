"""The config loader: layering, struct-mode refusals, MISSING, validators, shipped YAMLs."""
import glob

import pytest

from vdn_minimax_h3_b200.config import (ConfigError, InferenceConfig, StageA1Config, StageA2Config,
                                        StageBConfig, StageDMDConfig, load_config)
from vdn_minimax_h3_b200.config.schemas import (validate_ablation, validate_enums, validate_kernels,
                                                validate_parallel, validate_single_process,
                                                validate_stage_dmd)


def test_layering_and_dotlist():
    cfg = load_config(InferenceConfig, ["--config", "configs/inference/8nfe.yaml",
                                        "render.prompt_file=p.pt", "render.out=o.mp4",
                                        "render.seed=7", "precision.fp8.enabled=true"])
    assert cfg.render.num_steps == 8 and cfg.render.seed == 7 and cfg.precision.fp8.enabled


def test_refusals():
    with pytest.raises(ConfigError):
        load_config(InferenceConfig, ["render.prompt_file=p", "render.out=o", "render.nope=1"])
    with pytest.raises(ConfigError):
        load_config(InferenceConfig, ["render.out=o"])                 # prompt_file MISSING
    with pytest.raises(ConfigError):
        load_config(InferenceConfig, ["render.prompt_file=p", "render.out=o", "--bogus"])
    with pytest.raises(ConfigError):
        load_config(InferenceConfig, ["render.prompt_file=p", "render.out=o", "render.seed=x"])
    with pytest.raises(ConfigError):
        load_config(InferenceConfig, ["render.prompt_file=p", "render.out=o",
                                      "ablation.overrides={a: 1}"], (validate_ablation,))
    with pytest.raises(ConfigError):
        load_config(InferenceConfig, ["render.prompt_file=p", "render.out=o",
                                      "parallel.softmax_ranks=5"], (validate_single_process,))
    with pytest.raises(ConfigError):         # A2 has no model section
        load_config(StageA2Config, ["initialization.checkpoint=c", "data.index_file=i",
                                    "checkpoint.output_dir=o", "model.base.source=x"])


def test_shipped_yamls_load():
    extra = ["render.prompt_file=p", "render.out=o"]
    for path in glob.glob("configs/inference/*.yaml"):
        load_config(InferenceConfig, ["--config", path] + extra,
                    (validate_kernels, validate_parallel, validate_ablation))
    load_config(StageA1Config, ["--config", "configs/training/stage_a1_c1_vdn_anchor.yaml",
                                "data.index_file=i"], (validate_enums,))
    load_config(StageA2Config, ["--config", "configs/training/stage_a2_c1_vdn_anchor.yaml",
                                "data.index_file=i"])
    cfg = load_config(StageBConfig, ["--config", "configs/training/stage_b_c1_vdn_anchor.yaml",
                                     "data.index_file=i"])
    assert cfg.lora.rank == 64 and len(cfg.lora.targets) == 8
    load_config(StageDMDConfig, ["--config", "configs/training/stage_dmd_vdn.yaml",
                                 "data.index_file=i", "turbo.checkpoint=t"], (validate_stage_dmd,))
    with pytest.raises(ConfigError):
        load_config(StageDMDConfig, ["--config", "configs/training/stage_dmd_vdn.yaml",
                                     "data.index_file=i", "turbo.checkpoint=t",
                                     "dmd.fake_adapter_name=turbo"], (validate_stage_dmd,))
