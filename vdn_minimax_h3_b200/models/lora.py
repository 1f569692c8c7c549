"""Live LoRA adapters for training, with peft's parameter naming.

A targeted nn.Linear becomes a LoraLinear whose original layer is `base_layer` and whose
adapters are `lora_A[name]` / `lora_B[name]` (nn.ModuleDict), so state-dict keys read
`...to_q.lora_A.default.weight` exactly as the reference's peft-injected checkpoints do
(src/models/factory.py:61-121). Several named adapters can live on one layer; the ACTIVE
set is switched per forward (`set_active_adapters`) without touching requires_grad -- the
DMD roles (generator / real / fake) are switches of this set plus teacher_mode.
"""
import fnmatch
import math
import re

import torch
from torch import nn


class LoraLinear(nn.Module):
    def __init__(self, base: nn.Linear):
        super().__init__()
        self.base_layer = base
        self.lora_A = nn.ModuleDict()
        self.lora_B = nn.ModuleDict()
        self.scaling = {}
        self.active = []
        self.disabled = False

    @property
    def weight(self):
        return self.base_layer.weight

    @property
    def bias(self):
        return self.base_layer.bias

    @property
    def in_features(self):
        return self.base_layer.in_features

    @property
    def out_features(self):
        return self.base_layer.out_features

    def add_adapter(self, name, rank, alpha, init_b_zero=True):
        dev, dt = self.base_layer.weight.device, torch.float32
        a = nn.Linear(self.in_features, rank, bias=False, device=dev, dtype=dt)
        b = nn.Linear(rank, self.out_features, bias=False, device=dev, dtype=dt)
        nn.init.kaiming_uniform_(a.weight, a=math.sqrt(5))
        if init_b_zero:
            nn.init.zeros_(b.weight)
        self.lora_A[name] = a
        self.lora_B[name] = b
        self.scaling[name] = alpha / rank
        if name not in self.active:
            self.active.append(name)

    def forward(self, x):
        out = self.base_layer(x)
        if self.disabled:
            return out
        for name in self.active:
            if name in self.lora_A:
                a, b = self.lora_A[name], self.lora_B[name]
                out = out + (b(a(x.to(a.weight.dtype))) * self.scaling[name]).to(out.dtype)
        return out


def _matches(name, targets):
    for t in targets:
        if "*" in t:
            if fnmatch.fnmatch(name, "*" + t) or fnmatch.fnmatch(name, t):
                return True
        elif name.endswith(t):
            return True
    return False


def inject_lora(model, name, rank, alpha, targets, rank_pattern=None, alpha_pattern=None,
                init_b_zero=True):
    """Wrap every Linear whose module path ends with a target (glob allowed)."""
    rank_pattern, alpha_pattern = rank_pattern or {}, alpha_pattern or {}
    wrapped = 0
    for mod_name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            full = f"{mod_name}.{child_name}" if mod_name else child_name
            if not isinstance(child, (nn.Linear, LoraLinear)) or not _matches(full, targets):
                continue
            lin = child if isinstance(child, LoraLinear) else LoraLinear(child)
            r = next((v for k, v in rank_pattern.items() if re.search(k, full)), rank)
            al = next((v for k, v in alpha_pattern.items() if re.search(k, full)), alpha)
            lin.add_adapter(name, r, al, init_b_zero=init_b_zero)
            setattr(module, child_name, lin)
            wrapped += 1
    return wrapped


def lora_layers(model):
    return [m for m in model.modules() if isinstance(m, LoraLinear)]


def set_active_adapters(model, names):
    for m in lora_layers(model):
        m.active = [n for n in names if n in m.lora_A]


def set_adapters_enabled(model, enabled):
    for m in lora_layers(model):
        m.disabled = not enabled


def adapter_state(model, name):
    return {k: v for k, v in model.state_dict().items() if f".lora_A.{name}." in k or f".lora_B.{name}." in k}


def merge_and_unload(model):
    """Fold the active adapters into the base weights and put the plain Linears back."""
    for mod_name, module in list(model.named_modules()):
        for child_name, child in list(module.named_children()):
            if isinstance(child, LoraLinear):
                with torch.no_grad():
                    w = child.base_layer.weight
                    for n in child.active:
                        delta = child.lora_B[n].weight.float() @ child.lora_A[n].weight.float()
                        w.add_((delta * child.scaling[n]).to(w.dtype))
                setattr(module, child_name, child.base_layer)
    return model
