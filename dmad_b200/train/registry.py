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


class _IterationAdapter:
    """Trainer interface for models whose step is one whole DMAD iteration with their own optimisers
    and their own (synthetic or pooled) data: H3, EDM, SDXL."""

    def __init__(self, model, step_fn, modules: dict, optims: dict):
        self.model, self.step_fn = model, step_fn
        self.modules, self.optims = modules, optims

    def training_step(self, batch, it: int) -> dict:
        out = self.step_fn(batch, it)
        flat = {}
        for k, v in out.items():
            if isinstance(v, dict):
                flat.update({f"{k}/{kk}": vv for kk, vv in v.items()})
            else:
                flat[k] = v
        return flat

    def phase_of(self, it: int) -> str:
        return "all"

    def optimizers(self) -> dict:
        return {}

    def context_parallel_nets(self) -> list:
        return []

    @staticmethod
    def _per_rank(o) -> bool:
        """Optimisers whose state is this rank's shard (sharded data-parallel / FSDP) save per rank."""
        return hasattr(o, "layout") or hasattr(o, "blocks")

    def state_dicts(self):
        shared = {f"module/{k}": m.state_dict() for k, m in self.modules.items()}
        shared.update({f"optim/{k}": o.state_dict() for k, o in self.optims.items() if not self._per_rank(o)})
        per_rank = {f"optim/{k}": o.state_dict() for k, o in self.optims.items() if self._per_rank(o)}
        extra = getattr(self.model, "critic_state", None)
        if extra is not None:
            shared["critic_state"] = extra()
        ema = getattr(self.model, "ema_state", None)
        if ema is not None and ema() is not None:
            shared["ema_state"] = ema()
        return shared, (per_rank or None)

    def export_artifacts(self, ckpt_dir: str):
        """Extra files of a published checkpoint (rank 0): the H3 LoRA exports, the EDM generator EMAs."""
        fn = getattr(self.model, "export_loras", None) or getattr(self.model, "export_emas", None)
        if fn is not None:
            fn(ckpt_dir)

    def load_state_dicts(self, shared, per_rank):
        for k, m in self.modules.items():
            key = f"module/{k}"
            if key not in shared and k.startswith("ema_") and "module/generator" in shared:
                key = "module/generator"  # a checkpoint written before the EMAs were saved: restart them
            m.load_state_dict(shared[key])
        for k, o in self.optims.items():
            if self._per_rank(o):
                if not per_rank or f"optim/{k}" not in per_rank:
                    raise RuntimeError(f"checkpoint has no per-rank state of the sharded optimiser {k!r}")
                o.load_state_dict(per_rank[f"optim/{k}"])
            else:
                o.load_state_dict(shared[f"optim/{k}"])
        if "critic_state" in shared and hasattr(self.model, "load_critic_state"):
            self.model.load_critic_state(shared["critic_state"])
        if "ema_state" in shared and hasattr(self.model, "load_ema_state"):
            self.model.load_ema_state(shared["ema_state"])


def _dtype(device):
    return torch.bfloat16 if device.type == "cuda" else torch.float32


@register_model("h3_dmad")
def _build_h3(cfg: dict, device, seed: int):
    from ..distill.h3_dmad import H3DMAD, H3DMADConfig
    from ..models.h3 import H3Config
    from ..runtime.config import to_dataclass

    m = cfg.get("model", {})
    d = dict(m.get("distill") or {})
    net = m.get("net")
    hc = to_dataclass(H3DMADConfig, d)
    if isinstance(net, dict):
        hc.model = to_dataclass(H3Config, net)
    pool = None
    data = cfg.get("data", {})
    if data.get("kind") == "h3_pool":  # the prepared real / teacher / prompt-cache files
        from ..data.h3_pool import FileLatentPool
        pool = FileLatentPool(data["real_latent_dir"], hc.num_frames, data["caption_map"], data["prompt_cache"],
                              data["teacher_latent_dir"], seed=seed)
    model = H3DMAD(hc, device=device, pool=pool, dtype=_dtype(device), seed=seed)
    return _IterationAdapter(model, lambda batch, it: model.train_iteration(),
                             {"student": model.student, "fake": model.fake, "heads": model.heads},
                             {"student": model.opt_s, "fake": model.opt_f})


@register_model("edm_dmad")
def _build_edm(cfg: dict, device, seed: int):
    from ..distill.edm_dmad import EDMDMAD, EDMDMADConfig
    from ..runtime.config import to_dataclass

    m = cfg.get("model", {})
    ec = to_dataclass(EDMDMADConfig, dict(m.get("distill") or {}))
    torch.manual_seed(seed)
    model = EDMDMAD(ec, device=device)
    gen = torch.Generator().manual_seed(seed + 17)

    def step(batch, it):
        return model.train_step(batch if batch is not None else model.synthetic_batch(gen))
    modules = {"generator": model.generator, "critic": model.critic}
    modules.update({f"ema_{kimg:g}": ema for kimg, ema in model.emas.items()})  # saved, so a resume keeps them
    return _IterationAdapter(model, step, modules, {"generator": model.opt_g, "critic": model.opt_c})


@register_model("sdxl_dmad")
def _build_sdxl(cfg: dict, device, seed: int):
    from ..distill.sdxl_dmad import SDXLDMAD, SDXLDMADConfig
    from ..runtime.config import to_dataclass

    m = cfg.get("model", {})
    sc = to_dataclass(SDXLDMADConfig, dict(m.get("distill") or {}))
    model = SDXLDMAD(sc, device=device, dtype=_dtype(device), seed=seed)
    gen = torch.Generator().manual_seed(seed + 19)
    ucfg = sc.unet_kwargs or {}
    ctx_dim, pooled_dim = ucfg.get("ctx_dim", 2048), ucfg.get("pooled_dim", 1280)

    def step(batch, it):
        if batch is None:  # synthetic config-4 inputs: N(0,1) latents / text, uniform timesteps inside
            B, r = sc.batch_size, sc.latent
            dt = _dtype(device)
            batch = {"noise": torch.randn(B, 4, r, r, generator=gen).to(device),
                     "real": torch.randn(B, 4, r, r, generator=gen).to(device),
                     "teacher": torch.randn(B, 4, r, r, generator=gen).to(device),
                     "ctx": torch.randn(B, 77, ctx_dim, generator=gen).to(device, dt),
                     "pooled": torch.randn(B, pooled_dim, generator=gen).to(device, dt)}
        return model.train_step(batch)
    return _IterationAdapter(model, step, {"generator": model.generator, "critic": model.critic,
                                           "head_real": model.head_real, "head_teacher": model.head_teacher},
                             {"generator": model.opt_g, "critic": model.opt_c})
