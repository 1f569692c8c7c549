"""lr classes of the hybrid transform's parameters by module STRUCTURE (not name): small =
fixed-fan-in / vector parameters (alpha A_log, dt_bias, alpha.up, output_gate.up, branch norm,
short-conv taps), big = width-fan-in matrices. Reference parity: src/utils/lr_classes.py."""
from vdn_minimax_h3_b200.models.hybrid_transform import iter_hybrids


def lr_class_map(model):
    classes = {}
    for attn in iter_hybrids(model):
        for p in attn.parameters():
            classes[id(p)] = "big"
        lin = attn.linear_attention
        for p in (lin.alpha.A_log, lin.alpha.dt_bias, *lin.alpha.up.parameters(),
                  *lin.output_gate.up.parameters(), lin.norm.weight):
            classes[id(p)] = "small"
        if lin.short_conv is not None:
            for p in lin.short_conv.parameters():
                classes[id(p)] = "small"
        for p in attn.orig.parameters():
            classes.pop(id(p), None)
    return classes


def branch_lr_class_of(model, name, param):
    return lr_class_map(model).get(id(param), "big")
