"""Structured config sections and the per-entrypoint schemas (same YAML keys as the
reference's src/config/{common,inference,stage_a1,stage_a2,stage_b,stage_dmd}.py).

The three-layer rule holds: `model.*` is architecture (A1 only; it becomes the ModelSpec),
everything else configures one run, and `kernels` / `runtime` choices never enter a
checkpoint. Stages A2, B and DMD have no `model` section: their architecture comes from the
checkpoint, so an override attempt is an unknown key.
"""
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

from vdn_minimax_h3_b200.config.loader import MISSING

DELTA_RULES = ("sana_scaled", "vdn_solve", "vdn_scaled")
BRIDGES = ("alpha", "none")
SHORT_CONV_TARGETS = ("q", "k", "v")
ANCHOR_FRAME_MODES = ("none", "columns", "rows", "both")
SOFTMAX_BACKENDS = ("auto", "kernel", "ref", "flex", "decomposed")
REAL_SCORES = ("dense", "vdn")
VDN_ADAPTER_NAME = "default"
DEFAULT_LORA_TARGETS = (
    "attn.orig.to_q", "attn.orig.to_k", "attn.orig.to_v", "attn.orig.to_out.0",
    "token_refiner.refiner_blocks.*.attn.to_q", "token_refiner.refiner_blocks.*.attn.to_k",
    "token_refiner.refiner_blocks.*.attn.to_v", "token_refiner.refiner_blocks.*.attn.to_out.0",
)


# ------------------------------------------------------------------------- shared parts
@dataclass
class BaseModelConfig:
    library: str = "diffusers"
    class_name: str = "MiniMaxH3Transformer3DModel"
    source: str = MISSING
    subfolder: str = "transformer"
    revision: Optional[str] = None
    local_files_only: bool = True
    dtype: str = "bfloat16"
    config_overrides: Dict[str, Any] = field(default_factory=dict)


@dataclass
class SoftmaxAttentionConfig:
    radius: int = MISSING
    chunk: int = 0


@dataclass
class ShortConvConfig:
    targets: List[str] = field(default_factory=lambda: ["k", "v"])


@dataclass
class LinearAttentionConfig:
    delta_rule: str = MISSING
    linear_head_dim: Optional[int] = None
    bridge: str = "alpha"
    short_conv: ShortConvConfig = field(default_factory=ShortConvConfig)
    enable_text_state: bool = False
    a_fp32: bool = True


@dataclass
class HybridAttentionConfig:
    enable_softmax_gate: bool = True
    anchor_frames: str = "none"
    softmax_attention: SoftmaxAttentionConfig = field(default_factory=SoftmaxAttentionConfig)
    linear_attention: LinearAttentionConfig = field(default_factory=LinearAttentionConfig)


@dataclass
class ArchitectureConfig:
    hybrid_attention: HybridAttentionConfig = field(default_factory=HybridAttentionConfig)


@dataclass
class ModelConfig:
    base: BaseModelConfig = field(default_factory=BaseModelConfig)
    architecture: ArchitectureConfig = field(default_factory=ArchitectureConfig)


@dataclass
class DataConfig:
    index_file: str = MISSING
    num_workers: int = 4


@dataclass
class KernelsConfig:
    softmax_backend: str = "auto"


@dataclass
class RuntimeConfig:
    kernels: KernelsConfig = field(default_factory=KernelsConfig)
    # single-GPU inference: keep the DiT blocks in pinned host memory and stream each onto
    # the GPU while it runs (inference/offload.py; the reference's infer_diffusers
    # --offload_dit)
    offload_blocks: bool = False


@dataclass
class DistributedConfig:
    strategy: str = "fsdp"
    offload_activations: bool = False


@dataclass
class CheckpointConfig:
    output_dir: str = MISSING
    save_every: int = 50


def validate_enums(cfg):
    arch = getattr(getattr(cfg, "model", None), "architecture", None)
    if arch is None:
        return
    ha = arch.hybrid_attention
    if ha.linear_attention.delta_rule not in DELTA_RULES:
        raise ValueError(f"delta_rule {ha.linear_attention.delta_rule!r} not in {DELTA_RULES}")
    if ha.linear_attention.bridge not in BRIDGES:
        raise ValueError(f"bridge {ha.linear_attention.bridge!r} not in {BRIDGES}")
    t = list(ha.linear_attention.short_conv.targets)
    if any(x not in SHORT_CONV_TARGETS for x in t) or len(set(t)) != len(t):
        raise ValueError(f"short_conv.targets {t!r} must be a distinct subset of {SHORT_CONV_TARGETS}")
    if ha.anchor_frames not in ANCHOR_FRAME_MODES:
        raise ValueError(f"anchor_frames {ha.anchor_frames!r} not in {ANCHOR_FRAME_MODES}")


# ---------------------------------------------------------------------------- inference
@dataclass
class InferenceKernels(KernelsConfig):
    inference_kernels: bool = True


@dataclass
class Fp8Config:
    enabled: bool = False
    skip_end_blocks: int = 4


@dataclass
class PrecisionConfig:
    dtype: str = "bfloat16"
    fp8: Fp8Config = field(default_factory=Fp8Config)


@dataclass
class ParallelConfig:
    softmax_ranks: int = 0            # 0 = standard Ulysses; n = branch-parallel n + (world-n)
    tensor_parallel: int = 1          # TP group size (TP x Ulysses hybrid)
    exchange: str = "nccl"            # nccl | p2p (symmetric-memory peer kernels)
    profile: bool = False


@dataclass
class BehaviorConfig:
    teacher_mode: bool = False


@dataclass
class AblationConfig:
    enabled: bool = False
    overrides: Dict[str, Any] = field(default_factory=dict)


@dataclass
class RenderConfig:
    prompt_file: str = MISSING
    out: str = MISSING
    num_frames: int = 345
    num_steps: int = 50
    warmup_steps: int = 0
    seed: int = 42
    device: str = "cuda:0"
    video_shift: float = 12.0
    audio_shift: float = 3.0
    save_latents: bool = False
    latents_root: str = "artifacts/latents"
    record: bool = False


@dataclass
class ExternalLora:
    path: str = MISSING
    alpha: Optional[float] = None


@dataclass
class InferenceConfig:
    checkpoint: Optional[str] = None
    base_source: Optional[str] = None
    vae_source: Optional[str] = None
    synthetic_base: bool = False      # random-init backbone (no weights on disk)
    external_loras: List[ExternalLora] = field(default_factory=list)
    render: RenderConfig = field(default_factory=RenderConfig)
    kernels: InferenceKernels = field(default_factory=InferenceKernels)
    precision: PrecisionConfig = field(default_factory=PrecisionConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    behavior: BehaviorConfig = field(default_factory=BehaviorConfig)
    ablation: AblationConfig = field(default_factory=AblationConfig)


def validate_ablation(cfg):
    if cfg.ablation.overrides and not cfg.ablation.enabled:
        raise ValueError(f"semantic overrides {sorted(cfg.ablation.overrides)} require "
                         f"ablation.enabled=true -- they change what the model computes")


def validate_kernels(cfg):
    if cfg.kernels.softmax_backend not in SOFTMAX_BACKENDS:
        raise ValueError(f"kernels.softmax_backend {cfg.kernels.softmax_backend!r} not in {SOFTMAX_BACKENDS}")
    if cfg.kernels.inference_kernels and cfg.kernels.softmax_backend == "ref":
        raise ValueError("kernels.softmax_backend=ref is the eager oracle: it needs "
                         "kernels.inference_kernels=false (the fused engine runs the window kernel)")
    if not cfg.kernels.inference_kernels and cfg.precision.fp8.enabled:
        raise ValueError("precision.fp8 runs on the fused engine: it needs kernels.inference_kernels=true")
    if cfg.render.warmup_steps < 0:
        raise ValueError("render.warmup_steps must be >= 0")
    if cfg.precision.fp8.skip_end_blocks < 0:
        raise ValueError("precision.fp8.skip_end_blocks must be >= 0")


def validate_parallel(cfg):
    if cfg.parallel.softmax_ranks < 0:
        raise ValueError("parallel.softmax_ranks must be >= 0 (0 = standard Ulysses)")
    if cfg.parallel.tensor_parallel < 1:
        raise ValueError("parallel.tensor_parallel must be >= 1")
    if cfg.parallel.exchange not in ("nccl", "p2p"):
        raise ValueError("parallel.exchange must be nccl or p2p")


def validate_single_process(cfg):
    if asdict(cfg.parallel) != asdict(ParallelConfig()):
        raise ValueError("parallel.* only applies to the multi-GPU entrypoint (torchrun "
                         "infer_ulysses); infer is single-process")


# ------------------------------------------------------------------------------ stages
@dataclass
class A1Optimizer:
    name: str = "adamw"
    lr: float = 1.0e-4
    min_lr: float = 5.0e-6
    warmup_steps: int = 50
    weight_decay: float = 0.0
    grad_clip: float = 0.1
    big_lr_scale: float = 1.0
    small_lr_scale: float = 5.0
    small_eps: float = 2.0e-9


@dataclass
class A1Training:
    max_steps: int = 50
    gradient_accumulation_steps: int = 1
    seed: int = 0
    freeze_softmax_gate: bool = False
    per_layer_every: int = 25
    truncate_blocks: int = 0
    teacher_backend: str = "kernel"


@dataclass
class A1Checkpoint(CheckpointConfig):
    save_every: int = 25
    early_saves: List[int] = field(default_factory=lambda: [0, 1, 2, 4, 8])


@dataclass
class StageA1Config:
    model: ModelConfig = field(default_factory=ModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    training: A1Training = field(default_factory=A1Training)
    optimizer: A1Optimizer = field(default_factory=A1Optimizer)
    distributed: DistributedConfig = field(default_factory=DistributedConfig)
    checkpoint: A1Checkpoint = field(default_factory=A1Checkpoint)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)


@dataclass
class Initialization:
    checkpoint: str = MISSING
    base_source: Optional[str] = None


@dataclass
class A2Optimizer(A1Optimizer):
    warmup_steps: int = 25
    grad_clip: float = 1.0


@dataclass
class A2Training:
    max_steps: int = 100
    gradient_accumulation_steps: int = 1
    seed: int = 0
    audio_loss_weight: float = 1.0
    freeze_softmax_gate: bool = False
    ignore_stopped: bool = False
    auto_resume: bool = True


@dataclass
class FsdpDistributed:
    strategy: str = "fsdp2"
    activation_checkpointing: bool = True
    shard_size: int = 8
    offload_activations: bool = True
    memory_fraction: float = 0.92


@dataclass
class StateCheckpoint:
    output_dir: str = MISSING
    save_every: int = 10
    keep_states: int = 3
    early_saves: List[int] = field(default_factory=lambda: [0, 1, 2, 4, 8])


@dataclass
class StageA2Config:
    initialization: Initialization = field(default_factory=Initialization)
    data: DataConfig = field(default_factory=DataConfig)
    training: A2Training = field(default_factory=A2Training)
    optimizer: A2Optimizer = field(default_factory=A2Optimizer)
    distributed: FsdpDistributed = field(default_factory=FsdpDistributed)
    checkpoint: StateCheckpoint = field(default_factory=StateCheckpoint)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)


@dataclass
class LoraConfig:
    rank: int = 64
    alpha: int = 64
    targets: List[str] = field(default_factory=lambda: list(DEFAULT_LORA_TARGETS))


@dataclass
class BOptimizer:
    name: str = "adamw"
    lr: float = 1.0e-4
    min_lr: float = 5.0e-6
    warmup_steps: int = 100
    weight_decay: float = 0.0
    grad_clip: float = 1.0
    branch_lr_scale: float = 0.4
    small_lr_scale: float = 2.0
    small_eps: float = 2.0e-9


@dataclass
class BTraining:
    max_steps: int = 500
    gradient_accumulation_steps: int = 1
    seed: int = 0
    objective: str = "teacher"
    lambda_diffusion_video: float = 0.0
    lambda_diffusion_audio: float = 0.0
    audio_loss_weight: float = 1.0
    ignore_stopped: bool = False
    auto_resume: bool = True


@dataclass
class StageBConfig:
    initialization: Initialization = field(default_factory=Initialization)
    lora: Optional[LoraConfig] = None
    data: DataConfig = field(default_factory=DataConfig)
    training: BTraining = field(default_factory=BTraining)
    optimizer: BOptimizer = field(default_factory=BOptimizer)
    distributed: FsdpDistributed = field(default_factory=FsdpDistributed)
    checkpoint: StateCheckpoint = field(default_factory=StateCheckpoint)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)


@dataclass
class DInitialization(Initialization):
    source_step: int = 2000


@dataclass
class TurboConfig:
    checkpoint: str = MISSING
    adapter_name: str = "turbo"
    family: str = "external_v4_step600_ema"
    num_steps: int = 8
    video_shift: float = 12.0
    audio_shift: float = 3.0


@dataclass
class DMDConfig:
    real_score: str = "dense"
    fake_adapter_name: str = "fake"
    fake_rank: int = 128
    fake_updates_per_step: int = 3
    fake_warmup_steps: int = 10
    u_min: float = 0.02
    u_max: float = 0.98


@dataclass
class GenerationConfig:
    num_frames: int = 345
    latent_height: int = 48
    latent_width: int = 84


@dataclass
class DTraining:
    max_steps: int = 500
    seed: int = 0
    audio_loss_weight: float = 0.2
    ignore_stopped: bool = False
    auto_resume: bool = True


@dataclass
class DOptimizer:
    name: str = "adamw"
    lr: float = 1.0e-5
    min_lr: float = 1.0e-6
    warmup_steps: int = 100
    weight_decay: float = 0.0
    grad_clip: float = 1.0
    fake_lr: float = 2.0e-5
    fake_min_lr: float = 2.0e-6
    fake_warmup_steps: int = 10
    fake_grad_clip: float = 1.0


@dataclass
class StageDMDConfig:
    initialization: DInitialization = field(default_factory=DInitialization)
    turbo: TurboConfig = field(default_factory=TurboConfig)
    dmd: DMDConfig = field(default_factory=DMDConfig)
    generation: GenerationConfig = field(default_factory=GenerationConfig)
    data: DataConfig = field(default_factory=DataConfig)
    training: DTraining = field(default_factory=DTraining)
    optimizer: DOptimizer = field(default_factory=DOptimizer)
    distributed: FsdpDistributed = field(default_factory=FsdpDistributed)
    checkpoint: StateCheckpoint = field(default_factory=StateCheckpoint)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)


def validate_stage_dmd(cfg):
    if cfg.dmd.real_score not in REAL_SCORES:
        raise ValueError(f"dmd.real_score must be one of {REAL_SCORES}, got {cfg.dmd.real_score!r}")
    names = (cfg.turbo.adapter_name, cfg.dmd.fake_adapter_name)
    if len(set(names)) != 2 or VDN_ADAPTER_NAME in names:
        raise ValueError(f"turbo/fake adapter names must be distinct and neither may be "
                         f"{VDN_ADAPTER_NAME!r}; got {names}")
    if cfg.turbo.num_steps < 1:
        raise ValueError("turbo.num_steps must be >= 1")
    if cfg.turbo.video_shift <= 0 or cfg.turbo.audio_shift <= 0:
        raise ValueError("turbo shifts must be positive")
    if cfg.dmd.fake_rank < 1 or cfg.dmd.fake_updates_per_step < 1 or cfg.dmd.fake_warmup_steps < 0:
        raise ValueError("dmd.fake_rank >= 1, fake_updates_per_step >= 1, fake_warmup_steps >= 0")
