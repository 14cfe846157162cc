"""Typed experiment configs: YAML files + ``${env:VAR,default}`` interpolation + dotted overrides.

Parity: the H3 stack's YAML -> OmegaConf resolve -> plain dict (train/h3/lightx2v_train/runtime/
config.py:7-14, with ``${oc.env:WORLD_SIZE,1}``), and the Wan stack's experiment registry with
``experiment=<name>`` and ``key.sub=value`` overrides (train/wan/imaginaire/config.py:173-416,
train/wan/rcm/configs/registry_distill.py:27-98).

A config is a nested dict.  ``load_config(path, overrides)`` reads the YAML (``base:`` entries are
merged first, relative to the file), resolves interpolations, applies overrides (values parsed as
YAML scalars, so ``training.max_iters=10`` gives an int), and records ``config_path``.
``to_dataclass(cls, d)`` fills a dataclass (recursively) from a section and rejects unknown keys.
Experiments registered with ``register_experiment(name, dict)`` are selected with
``experiment=<name>`` (merged before the other overrides).
"""
from __future__ import annotations

import copy
import dataclasses
import os
import re
import typing
from typing import Any

import yaml

_EXPERIMENTS: dict[str, dict] = {}
_ENV = re.compile(r"\$\{(?:oc\.)?env:([A-Za-z_][A-Za-z0-9_]*)(?:,([^}]*))?\}")


def register_experiment(name: str, cfg: dict):
    _EXPERIMENTS[name] = copy.deepcopy(cfg)


def experiments() -> list[str]:
    return sorted(_EXPERIMENTS)


def experiment(name: str) -> dict:
    """A copy of a registered experiment's overrides."""
    return copy.deepcopy(_EXPERIMENTS[name])


def merge(base: dict, over: dict) -> dict:
    """Recursive dict merge (``over`` wins; dicts merge, everything else replaces)."""
    out = copy.deepcopy(base)
    for k, v in over.items():
        if isinstance(v, dict) and isinstance(out.get(k), dict):
            out[k] = merge(out[k], v)
        else:
            out[k] = copy.deepcopy(v)
    return out


def _resolve(v):
    if isinstance(v, dict):
        return {k: _resolve(x) for k, x in v.items()}
    if isinstance(v, list):
        return [_resolve(x) for x in v]
    if isinstance(v, str):
        m = _ENV.fullmatch(v.strip())
        if m:  # whole-string interpolation keeps the YAML type of the value
            raw = os.environ.get(m.group(1), m.group(2) if m.group(2) is not None else "")
            return parse_scalar(raw) if raw != "" else raw
        return _ENV.sub(lambda mm: os.environ.get(mm.group(1), mm.group(2) or ""), v)
    return v


def set_dotted(cfg: dict, key: str, value):
    parts = key.split(".")
    d = cfg
    for p in parts[:-1]:
        if p not in d or not isinstance(d[p], dict):
            d[p] = {}
        d = d[p]
    d[parts[-1]] = value


def get_dotted(cfg: dict, key: str, default=None):
    d = cfg
    for p in key.split("."):
        if not isinstance(d, dict) or p not in d:
            return default
        d = d[p]
    return d


def parse_scalar(v: str):
    """YAML value of an override; also accepts floats YAML 1.1 leaves as strings (``2e-6``)."""
    if v.strip() == "":
        return None
    x = yaml.safe_load(v)
    if isinstance(x, str):
        try:
            return float(x)
        except ValueError:
            return x
    return x


def parse_overrides(items: list[str]) -> list[tuple[str, Any]]:
    out = []
    for it in items:
        if "=" not in it:
            raise ValueError(f"override {it!r} is not key=value")
        k, v = it.split("=", 1)
        out.append((k.strip(), parse_scalar(v)))
    return out


def _read_yaml(path: str, seen=()) -> dict:
    path = os.path.abspath(path)
    if path in seen:
        raise ValueError(f"config base cycle through {path}")
    with open(path) as f:
        d = yaml.safe_load(f) or {}
    bases = d.pop("base", None)
    if bases:
        out: dict = {}
        for b in [bases] if isinstance(bases, str) else bases:
            out = merge(out, _read_yaml(os.path.join(os.path.dirname(path), b), seen + (path,)))
        d = merge(out, d)
    return d


def load_config(path: str | None = None, overrides: list[str] | None = None, base: dict | None = None) -> dict:
    cfg = copy.deepcopy(base) if base else {}
    if path:
        cfg = merge(cfg, _read_yaml(path))
        cfg["config_path"] = os.path.abspath(path)
    ovs = parse_overrides(overrides or [])
    for k, v in ovs:
        if k == "experiment":
            if v not in _EXPERIMENTS:
                raise KeyError(f"unknown experiment {v!r}; registered: {experiments()}")
            cfg = merge(cfg, _EXPERIMENTS[v])
            cfg["experiment"] = v
    for k, v in ovs:
        if k != "experiment":
            set_dotted(cfg, k, v)
    return _resolve(cfg)


def save_config(cfg: dict, path: str):
    with open(path, "w") as f:
        yaml.safe_dump(_plain(cfg), f, sort_keys=False)


def _plain(v):
    if dataclasses.is_dataclass(v):
        return _plain(dataclasses.asdict(v))
    if isinstance(v, dict):
        return {k: _plain(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_plain(x) for x in v]
    return v


def to_dataclass(cls, d: dict | None, strict: bool = True):
    """Build ``cls`` from dict ``d``; nested dataclass fields are built recursively, tuples coerced."""
    d = dict(d or {})
    hints = typing.get_type_hints(cls)
    kw = {}
    names = {f.name for f in dataclasses.fields(cls)}
    unknown = set(d) - names
    if unknown and strict:
        raise KeyError(f"{cls.__name__}: unknown config keys {sorted(unknown)}")
    for f in dataclasses.fields(cls):
        if f.name not in d:
            continue
        v = d[f.name]
        t = hints.get(f.name)
        sub = _dataclass_type(t)
        if sub is not None and isinstance(v, dict):
            v = to_dataclass(sub, v, strict)
        elif isinstance(v, list) and _is_tuple(t):
            v = tuple(v)
        kw[f.name] = v
    return cls(**kw)


def _dataclass_type(t):
    if dataclasses.is_dataclass(t):
        return t
    for a in typing.get_args(t) or ():
        if dataclasses.is_dataclass(a):
            return a
    return None


def _is_tuple(t):
    if t is tuple or typing.get_origin(t) is tuple:
        return True
    return any(a is tuple or typing.get_origin(a) is tuple for a in typing.get_args(t) or ())
