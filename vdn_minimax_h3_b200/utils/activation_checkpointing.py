"""Two-level activation checkpointing: each DiT block as a whole and, inside it, the
attention and the feed-forward as separate regions (reference
src/utils/activation_checkpointing.py:27-64). Non-reentrant checkpoints, installed as
instance-level forward wrappers so the module tree and parameter names are unchanged."""
import functools
import types

import torch
from torch.utils.checkpoint import checkpoint


def checkpoint_forward(module):
    if getattr(module, "_vdn_ckpt", False):
        return module
    inner = module.forward

    @functools.wraps(inner)
    def forward(*args, **kwargs):
        if not torch.is_grad_enabled():
            return inner(*args, **kwargs)
        return checkpoint(inner, *args, use_reentrant=False, **kwargs)

    module.forward = forward
    module._vdn_ckpt = True
    return module


def split_block_checkpoints(model, parts=("attn", "ff")):
    """Checkpoint each block's sub-layers (the inner level)."""
    n = 0
    for block in model.transformer_blocks:
        for name in parts:
            sub = getattr(block, name, None)
            if sub is not None:
                checkpoint_forward(sub)
                n += 1
    return n


def enable_block_checkpointing(model, split=True):
    if split:
        split_block_checkpoints(model)
    for block in model.transformer_blocks:
        checkpoint_forward(block)
    return model
