"""One loader for every entrypoint: structured dataclass defaults < YAML files < CLI dotlist.

    cfg = load_config(InferenceConfig, argv, extra_validators=(...))

The control surface is exactly three flags -- --config (repeatable), --print-config,
--validate-only -- plus `a.b.c=value` overrides, as in the reference
(src/config/loader.py:21-86). Struct semantics: an unknown key in any layer is an error
naming its full path; a field left at MISSING ("???") after merging is an error; values are
checked against the field types. Implemented on dataclasses + PyYAML (no OmegaConf).
"""
import argparse
import copy
import dataclasses
import sys
import typing
from typing import Any, Callable, Dict, Optional, Sequence

import yaml

MISSING = "???"


class ConfigError(SystemExit):
    def __init__(self, message):
        super().__init__(f"config error: {message}")


def _origin(tp):
    return typing.get_origin(tp)


def _is_optional(tp):
    return _origin(tp) is typing.Union and type(None) in typing.get_args(tp)


def _inner(tp):
    if _is_optional(tp):
        args = [a for a in typing.get_args(tp) if a is not type(None)]
        return args[0]
    return tp


def _coerce(value, tp, path):
    if value is None:
        if _is_optional(tp) or tp is Any:
            return None
        raise ConfigError(f"{path}: None is not allowed for a non-optional field")
    if isinstance(value, str) and value == MISSING:
        return value
    tp = _inner(tp)
    if tp is Any:
        return value
    if dataclasses.is_dataclass(tp):
        if dataclasses.is_dataclass(value):
            return value
        if not isinstance(value, dict):
            raise ConfigError(f"{path}: expected a mapping for {tp.__name__}")
        return _merge(_default(tp), value, path)
    org = _origin(tp)
    if org in (list, typing.List):
        (sub,) = typing.get_args(tp) or (Any,)
        if not isinstance(value, (list, tuple)):
            raise ConfigError(f"{path}: expected a list")
        return [_coerce(v, sub, f"{path}[{i}]") for i, v in enumerate(value)]
    if org in (dict, typing.Dict):
        if not isinstance(value, dict):
            raise ConfigError(f"{path}: expected a mapping")
        return dict(value)
    if tp is bool:
        if isinstance(value, bool):
            return value
        raise ConfigError(f"{path}: expected a bool, got {value!r}")
    if tp is int:
        if isinstance(value, bool) or not isinstance(value, int):
            raise ConfigError(f"{path}: expected an int, got {value!r}")
        return value
    if tp is float:
        if isinstance(value, str):
            try:                      # YAML 1.1 reads "1e-6" (no dot) as a string
                return float(value)
            except ValueError:
                pass
        if isinstance(value, bool) or not isinstance(value, (int, float)):
            raise ConfigError(f"{path}: expected a float, got {value!r}")
        return float(value)
    if tp is str:
        if not isinstance(value, str):
            raise ConfigError(f"{path}: expected a string, got {value!r}")
        return value
    return value


def _default(cls):
    return cls()


def _merge(obj, patch: Dict[str, Any], path=""):
    """A copy of dataclass `obj` with the mapping `patch` merged in (struct mode)."""
    obj = copy.deepcopy(obj)
    hints = typing.get_type_hints(type(obj))
    names = {f.name for f in dataclasses.fields(obj)}
    for key, value in patch.items():
        full = f"{path}.{key}" if path else key
        if key not in names:
            raise ConfigError(f"unknown key {full!r}")
        tp = hints[key]
        cur = getattr(obj, key)
        inner = _inner(tp)
        if dataclasses.is_dataclass(inner) and isinstance(value, dict):
            base = cur if dataclasses.is_dataclass(cur) else _default(inner)
            setattr(obj, key, _merge(base, value, full))
        else:
            setattr(obj, key, _coerce(value, tp, full))
    return obj


def _set_path(tree: Dict[str, Any], dotted: str, value):
    parts = dotted.split(".")
    node = tree
    for p in parts[:-1]:
        node = node.setdefault(p, {})
    node[parts[-1]] = value


def _missing(obj, path=""):
    out = []
    for f in dataclasses.fields(obj):
        v = getattr(obj, f.name)
        full = f"{path}.{f.name}" if path else f.name
        if isinstance(v, str) and v == MISSING:
            out.append(full)
        elif dataclasses.is_dataclass(v):
            out.extend(_missing(v, full))
    return out


def to_dict(cfg):
    return dataclasses.asdict(cfg)


def resolved_dict(cfg):
    """Plain-dict snapshot (stamped into train states as resolved_training_config)."""
    return to_dict(cfg)


def merge(cfg, patch: Dict[str, Any]):
    return _merge(cfg, patch)


def load_config(schema_cls, argv: Optional[Sequence[str]] = None,
                extra_validators: Sequence[Callable[[Any], None]] = ()):
    parser = argparse.ArgumentParser(add_help=True)
    parser.add_argument("--config", action="append", default=[])
    parser.add_argument("--print-config", action="store_true")
    parser.add_argument("--validate-only", action="store_true")
    args, dotlist = parser.parse_known_args(argv)
    bad = [d for d in dotlist if d.startswith("--")]
    if bad:
        raise ConfigError(f"unknown flag(s) {bad}; only --config / --print-config / "
                          f"--validate-only exist -- everything else is a dotlist override")
    cfg = schema_cls()
    for path in args.config:
        with open(path) as f:
            data = yaml.safe_load(f) or {}
        cfg = _merge(cfg, data)
    if dotlist:
        patch = {}
        for item in dotlist:
            if "=" not in item:
                raise ConfigError(f"override {item!r} is not key=value")
            k, v = item.split("=", 1)
            _set_path(patch, k, yaml.safe_load(v) if v != "" else "")
        cfg = _merge(cfg, patch)
    missing = _missing(cfg)
    if missing:
        raise ConfigError(f"missing mandatory value(s): {missing}")
    for validate in extra_validators:
        try:
            validate(cfg)
        except ValueError as exc:
            raise ConfigError(str(exc)) from exc
    if args.print_config:
        print(yaml.safe_dump(to_dict(cfg), sort_keys=False), end="")
        sys.exit(0)
    if args.validate_only:
        print("config ok", file=sys.stderr)
        sys.exit(0)
    return cfg
