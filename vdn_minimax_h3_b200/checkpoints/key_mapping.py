"""Pre-v2 -> v2 renames of checkpoint keys and transform-config fields, and the value
registries the config schema and the ModelSpec share.

Reference parity: src/checkpoints/key_mapping.py:15-102. The rename TABLE has to be the
reference's (it is a file-format fact: older checkpoints spell their keys this way), so
the rules and their first-match-wins order are kept as they are.
"""
KEY_RULES = (
    (".attn.far.gate.", ".attn.linear_attention.output_gate."),
    (".attn.far.", ".attn.linear_attention."),
    (".attn.local_gate.", ".attn.softmax_gate."),
    (".attn.w_o_far.", ".attn.to_out_linear."),
)
META_KEYS = ("__window__", "__branch__", "__truncated__")
CONFIG_FIELD_RENAMES = {
    "backend": "delta_rule",
    "far_head_dim": "linear_head_dim",
    "use_local_mass_gate": "enable_softmax_gate",
    "text_state": "enable_text_state",
    "w_o_far_scale": None,
}
DELTA_RULE_VALUES = ("sana_scaled", "vdn_solve", "vdn_scaled")
SHORT_CONV_TARGETS = ("q", "k", "v")
SHORT_CONV_VALUES = {False: [], "sep": ["k", "v"]}
ANCHOR_FRAME_MODES = ("none", "columns", "rows", "both")


def map_key(name: str) -> str:
    if name in META_KEYS:
        return name
    for old, new in KEY_RULES:
        if old in name:
            return name.replace(old, new, 1)
    return name


def map_keys(names):
    out = {n: map_key(n) for n in names}
    seen = {}
    for old, new in out.items():
        if new in seen:
            raise ValueError(f"key collision: {old!r} and {seen[new]!r} both map to {new!r}")
        seen[new] = old
    return out


def map_config(config: dict) -> dict:
    out = {}
    for key, value in config.items():
        new = CONFIG_FIELD_RENAMES.get(key, key)
        if new is not None:
            out[new] = value
    if "short_conv" in out:
        v = out["short_conv"]
        if isinstance(v, dict):
            targets = list(v["targets"])
        elif isinstance(v, (list, tuple)):
            targets = list(v)
        elif v is True:
            raise ValueError("short_conv=True is the dense 5^3 depthwise conv, which is not "
                             "implemented")
        else:
            targets = SHORT_CONV_VALUES[v]
        out["short_conv"] = {"targets": targets}
    if "anchor_frames" in out:
        mode = out["anchor_frames"]
        if isinstance(mode, bool):
            mode = "both" if mode else "none"
        if mode not in ANCHOR_FRAME_MODES:
            raise ValueError(f"unknown anchor_frames {mode!r}")
        out["anchor_frames"] = mode
    rule = out.get("delta_rule")
    if rule is not None and rule not in DELTA_RULE_VALUES:
        raise ValueError(f"unknown delta_rule {rule!r}")
    return out
