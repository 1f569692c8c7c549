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
    names = set()
    for path in glob.glob("configs/inference/*.yaml"):
        cfg = load_config(InferenceConfig, ["--config", path] + extra,
                          (validate_kernels, validate_parallel, validate_ablation))
        name = path.rsplit("/", 1)[-1]
        names.add(name)
        # the ladder: rung 0 is the eager model, `_tuned` the fused engine, `_fp8` adds fp8
        assert cfg.kernels.inference_kernels == ("_tuned" in name), name
        assert cfg.precision.fp8.enabled == ("_fp8" in name), name
        assert (cfg.parallel.tensor_parallel > 1 or cfg.parallel.softmax_ranks > 0) == ("_b200" in name)
    assert {"8nfe.yaml", "8nfe_tuned.yaml", "8nfe_tuned_fp8.yaml", "8nfe_tuned_fp8_ulysses_b200.yaml",
            "50nfe.yaml", "50nfe_tuned.yaml", "50nfe_tuned_fp8.yaml"} <= names
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


def test_kernel_settings_that_cannot_run_are_refused():
    base = ["render.prompt_file=p", "render.out=o"]
    with pytest.raises(ConfigError):      # the eager oracle is not the fused engine's path
        load_config(InferenceConfig, base + ["kernels.softmax_backend=ref"], (validate_kernels,))
    with pytest.raises(ConfigError):      # fp8 Linears exist only in the fused engine
        load_config(InferenceConfig, base + ["kernels.inference_kernels=false",
                                             "precision.fp8.enabled=true"], (validate_kernels,))
    cfg = load_config(InferenceConfig, base + ["kernels.inference_kernels=false",
                                               "kernels.softmax_backend=ref"], (validate_kernels,))
    assert cfg.kernels.softmax_backend == "ref"


def test_softmax_backend_names():
    """The reference's backend names map onto this build's paths; unknown names are refused."""
    from vdn_minimax_h3_b200.models.factory import TINY_HYBRID, build_model, make_spec
    from vdn_minimax_h3_b200.models.h3 import h3_tiny_config
    from vdn_minimax_h3_b200.models.hybrid_transform import iter_hybrids, set_softmax_backend
    model = build_model(make_spec(h3_tiny_config(), TINY_HYBRID, dtype="float32"), init="random")
    for name, impl in (("flex", "kernel"), ("decomposed", "kernel"), ("ref", "ref"), ("auto", "auto")):
        assert set_softmax_backend(model, name) == impl
        assert all(a.softmax_impl == impl for a in iter_hybrids(model))
    with pytest.raises(ValueError):
        set_softmax_backend(model, "triton")
