"""Entry of the exported component: `VDNMiniMaxH3Transformer3DModel.from_pretrained(dir)`.

Reference parity: src/diffusers_export/modeling.py:117-288 (a component class whose
`from_pretrained` assembles the base transformer, the hybrid branch weights and the
checkpoint's adapters from the paths in the component's config.json). The exporter
(export/component.py) flattens this module and the model code it imports into one
`modeling_vdn_h3.py`; this source is also importable in place.
"""
import json
import os

import torch
from torch import nn

from vdn_minimax_h3_b200.checkpoints.export_dir import load_checkpoint_dir
from vdn_minimax_h3_b200.inference.lora import merge_lora_state
from vdn_minimax_h3_b200.models.factory import build_model, load_model_weights
from vdn_minimax_h3_b200.models.hybrid_transform import iter_hybrids

COMPONENT_CONFIG = "config.json"
COMPONENT_CLASS = "VDNMiniMaxH3Transformer3DModel"


class VDNMiniMaxH3Transformer3DModel(nn.Module):
    """The hybrid VDN-H3 transformer assembled from a component directory."""

    def __init__(self, model, config):
        super().__init__()
        self.transformer = model
        self.config = config

    @classmethod
    def from_pretrained(cls, path, subfolder=None, device="cpu", base_source=None,
                        random_base_seed=None):
        """config.json's `vdn` block names the checkpoint (relative to the component) and
        the base weights; `random_base_seed` builds a random backbone instead (no base
        weights offline). Branch weights load strictly; adapters merge into the base."""
        root = os.path.join(path, subfolder) if subfolder else path
        with open(os.path.join(root, COMPONENT_CONFIG)) as f:
            config = json.load(f)
        if config.get("_class_name") != COMPONENT_CLASS:
            raise ValueError(f"{root}: not a {COMPONENT_CLASS} component")
        vdn = config["vdn"]
        ckpt = os.path.normpath(os.path.join(root, vdn.get("checkpoint", "..")))
        artifact = load_checkpoint_dir(ckpt)
        init = "random" if random_base_seed is not None else "load"
        base = vdn.get("base") or {}
        model = build_model(artifact.model_spec, device=device, init=init,
                            base_source=base_source or base.get("source"),
                            seed=random_base_seed or 0)
        branch = {k: v for k, v in artifact.weights.items() if ".lora_" not in k}
        lora = {k: v for k, v in artifact.weights.items() if ".lora_" in k}
        load_model_weights(model, branch)
        if lora:
            scale = 1.0
            for a in artifact.model_spec.get("adapters", []):
                c = a.get("config", {})
                if "alpha" in c and "rank" in c:
                    scale = float(c["alpha"]) / float(c["rank"])
            merge_lora_state(model, lora, scale=scale)
        dtype = getattr(torch, vdn.get("branch_dtype", "bfloat16"))
        for attn in iter_hybrids(model):
            attn.to(dtype)
            attn.linear_attention.alpha.float()
        model.eval()
        return cls(model, config)

    def forward(self, *args, **kwargs):
        return self.transformer(*args, **kwargs)
