"""The hybrid transform: dense H3 in, softmax + linear hybrid out, plus runtime setters.

Reference parity: src/models/hybrid_transform.py:19-156. Each DiT block's `.attn` is
swapped for a HybridAttention wrapping (and reusing) the original module, so the teacher is
always `attn.orig`; the token refiner is never converted.
"""
from vdn_minimax_h3_b200.models.hybrid_attention import SOFTMAX_BACKENDS, HybridAttention

TRANSFORM_TYPE = "hybrid_attention"
TRANSFORM_VERSION = 2


def apply_hybrid_attention_transform(model, config: dict):
    """`config` is the resolved (nested v2) transform config of a ModelSpec."""
    soft = config["softmax_attention"]
    lin = dict(config["linear_attention"])
    short_conv = tuple(lin.pop("short_conv")["targets"])
    hidden = model.config.hidden_size
    hybrids = []
    for block in model.transformer_blocks:
        dev = block.attn.to_q.weight.device
        import torch
        with torch.device(dev):
            hybrid = HybridAttention(
                block.attn, hidden_size=hidden, delta_rule=lin["delta_rule"],
                linear_head_dim=lin["linear_head_dim"], bridge=lin["bridge"],
                a_fp32=lin["a_fp32"], short_conv=short_conv,
                enable_text_state=lin["enable_text_state"], radius=soft["radius"],
                chunk=soft["chunk"], anchor_frames=config["anchor_frames"],
                enable_softmax_gate=config["enable_softmax_gate"])
        block.attn = hybrid
        hybrids.append(hybrid)
    return hybrids


def iter_hybrids(model):
    for block in model.transformer_blocks:
        if isinstance(block.attn, HybridAttention):
            yield block.attn


def set_layout(model, layout):
    for attn in iter_hybrids(model):
        attn.layout = layout


def set_teacher_mode(model, enabled: bool):
    for attn in iter_hybrids(model):
        attn.teacher_mode = enabled


# The reference's backend names: `flex` (FlexAttention / FA4) and `decomposed` (FA4 varlen
# + cuDNN legs) are both its GPU window paths; here both are the sm_100a window kernel.
BACKEND_ALIASES = {"auto": "auto", "kernel": "kernel", "flex": "kernel", "decomposed": "kernel",
                   "ref": "ref"}


def set_softmax_backend(model, backend: str) -> str:
    """auto (the sm_100a window kernel where its tensors qualify, else the oracle) | kernel
    (the kernel required on CUDA; `flex` and `decomposed` mean the same) | ref (the eager
    per-segment oracle even on CUDA). Returns the backend the hybrids now use."""
    impl = BACKEND_ALIASES.get(backend)
    if impl is None or impl not in SOFTMAX_BACKENDS:
        raise ValueError(f"softmax_backend={backend!r}; expected one of {sorted(BACKEND_ALIASES)}")
    for attn in iter_hybrids(model):
        attn.softmax_impl = impl
    return impl


def set_inference_mode(model, enabled: bool):
    for attn in iter_hybrids(model):
        attn.inference_mode = enabled


def is_transform_parameter(name: str) -> bool:
    """Parameter NAMES the transform introduced (branch, gates, to_out_linear on a DiT
    block): not `.attn.orig.*`, not the refiner, not LoRA."""
    return (".attn." in name and ".attn.orig." not in name
            and "token_refiner" not in name and "lora_" not in name)


def hybrid_new_parameters(model):
    out = []
    for index, block in enumerate(model.transformer_blocks):
        attn = block.attn
        if not isinstance(attn, HybridAttention):
            continue
        out.append((index, [(f"transformer_blocks.{index}.attn.{n}", p)
                            for n, p in attn.named_parameters() if not n.startswith("orig.")]))
    return out


def transform_config_of_model(model) -> dict:
    attn = next(iter_hybrids(model), None)
    if attn is None:
        raise ValueError("model carries no HybridAttention -- nothing to stamp")
    lin = attn.linear_attention
    return dict(
        enable_softmax_gate=attn.enable_softmax_gate, anchor_frames=attn.anchor_frames,
        softmax_attention=dict(radius=attn.radius, chunk=attn.chunk),
        linear_attention=dict(
            delta_rule=lin.delta_rule, bridge=lin.bridge, linear_head_dim=lin.head_dim,
            a_fp32=lin.a_fp32,
            short_conv=dict(targets=list(lin.short_conv.projs) if lin.short_conv else []),
            enable_text_state=attn.enable_text_state))
