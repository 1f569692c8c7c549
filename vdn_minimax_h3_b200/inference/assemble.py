"""Inference assembly: spec -> base -> hybrid transform -> branch weights -> LoRA merges ->
dtype policy -> (optional fp8) -> the fused-kernel InferenceEngine.

Reference parity: src/inference/utils/assemble.py:101-203 (build_inference_model and the
render record). The order matters for the same reasons it does there: adapters merge into
the bf16 base before anything packs or quantises the weights, and the engine packing is
one-way.
"""
import time

import torch

from vdn_minimax_h3_b200.inference.engine import InferenceEngine
from vdn_minimax_h3_b200.inference.lora import merge_lora_state, random_lora_state
from vdn_minimax_h3_b200.models.factory import RELEASED_HYBRID, build_model, load_model_weights, make_spec
from vdn_minimax_h3_b200.models.h3 import H3Config, h3_full_config
from vdn_minimax_h3_b200.models.hybrid_transform import iter_hybrids


def cast_branch_for_inference(model, dtype=torch.bfloat16):
    """Branch parameters to the compute dtype, except FrameKDAAlpha (a deliberate fp32
    island, reference linear_attention/layers.py:47-69)."""
    for attn in iter_hybrids(model):
        attn.to(dtype)
        attn.linear_attention.alpha.float()


def build_synthetic_model(cfg: H3Config = None, hybrid=RELEASED_HYBRID, device="cuda", seed=0,
                          lora_ranks=(("default", 64), ("turbo", 64))):
    """The full-geometry VDN-H3 with random weights (nothing is downloaded): random backbone,
    random branch, random `default`/`turbo` adapters merged at load."""
    cfg = cfg or h3_full_config()
    spec = make_spec(cfg, hybrid)
    torch.manual_seed(seed)
    t0 = time.perf_counter()
    model = build_model(spec, device=device, init="random", seed=seed)
    for i, (name, rank) in enumerate(lora_ranks):
        state = random_lora_state(model, rank, seed=seed + 1 + i, name=name, device=device)
        merge_lora_state(model, state, scale=1.0)
        del state
    cast_branch_for_inference(model)
    model.eval()
    return model, time.perf_counter() - t0


def build_inference_engine(model, fp8=False):
    """The fused-kernel engine; fp8=True quantises the QKV / FF projections to block-scaled
    E4M3 once here (the reference's assembly step 'fp8', assemble.py:101-180)."""
    return InferenceEngine(model, fp8=fp8)


def build_from_checkpoint(artifact, device="cuda", base_source=None, init="load"):
    """A v2 checkpoint artifact -> canonical model with its branch weights and merged LoRA."""
    model = build_model(artifact.model_spec, device=device, base_source=base_source, init=init)
    branch = {k: v for k, v in artifact.weights.items() if ".lora_" not in k}
    lora = {k: v for k, v in artifact.weights.items() if ".lora_" in k}
    load_model_weights(model, branch)
    if lora:
        scale = 1.0
        for a in artifact.model_spec.get("adapters", []):
            cfg = a["config"]
            if "alpha" in cfg and "rank" in cfg:
                scale = float(cfg["alpha"]) / float(cfg["rank"])
        merge_lora_state(model, lora, scale=scale)
    cast_branch_for_inference(model)
    model.eval()
    return model
