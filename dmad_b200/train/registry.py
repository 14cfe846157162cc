"""Model registry with lazy construction by name.

Parity: the H3 stack's model / trainer registries with lazy import by name
(train/h3/lightx2v_train/utils/registry.py:5-126) and the Wan experiment registry
(train/wan/rcm/configs/registry_distill.py:27-98).  A builder takes the whole config dict, the
device and a seed and returns an object with ``training_step(batch, it)``, ``phase_of(it)``,
``optimizers()``, ``state_dicts()`` / ``load_state_dicts()`` and ``context_parallel_nets()``.
"""
from __future__ import annotations

from typing import Callable

import torch

_MODELS: dict[str, Callable] = {}


def register_model(name: str):
    def deco(fn):
        _MODELS[name] = fn
        return fn
    return deco


def registered_models() -> list[str]:
    return sorted(_MODELS)


def build_model(cfg: dict, device, seed: int = 0):
    fam = cfg.get("model", {}).get("family", "wan_dmad")
    if fam not in _MODELS:
        raise KeyError(f"unknown model family {fam!r}; registered: {registered_models()}")
    return _MODELS[fam](cfg, torch.device(device), seed)


@register_model("wan_dmad")
def _build_wan_dmad(cfg: dict, device, seed: int):
    from ..distill.wan_dmad import WanDMAD, WanDMADConfig
    from ..models.wan import WanConfig, wan_config
    from ..runtime.config import to_dataclass

    m = cfg.get("model", {})
    net = m.get("net", "wan2.1-1.3b")
    if isinstance(net, str):
        net_cfg = wan_config(net)
    else:
        net = dict(net)
        base = net.pop("name", None)
        net_cfg = wan_config(base, **net) if base else to_dataclass(WanConfig, net)
    dcfg = to_dataclass(WanDMADConfig, {k: v for k, v in (m.get("distill") or {}).items()})
    dcfg.net = net_cfg
    par = cfg.get("parallel", {})
    if "dp_optimizer" in par:
        dcfg.dp_optimizer = par["dp_optimizer"]
    dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
    return WanDMAD(dcfg, device=device, dtype=dtype, seed=seed)
