"""DMAD for the SDXL-shaped U-Net.

Parity with train/image/main/sd_guidance.py and sd_unified_model.py:
* generator: epsilon-prediction U-Net; 4-step ``denoising_step_list`` (999, 749, 499, 249); backward
  simulation runs the generator's own sampler for a random number of steps (shared across ranks) and
  re-noises to the selected step; the pure-noise step starts from noise; x0 = (x_t - sqrt(1-a) eps)/sqrt(a);
* critic: a copy of the U-Net with the decoder removed (bottleneck [N, 1280, H/4, W/4]), two conv heads
  (three stride-2 convs, a 4x4/stride-4 conv, a 1x1 conv), frozen-gain spectral norm on every trainable
  conv (200 power iterations at set-up); DDPM noising at t ~ U[0, critic_max_timestep), one t per sample
  index shared by T / G / Q; gap bands t // 100, all-reduced;
* one iteration = generator update then critic update on the same generated batch.
"""
from __future__ import annotations

import copy
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F
from ..algorithms.dmad import NUM_GAP_BANDS
from ..algorithms.spectral import apply_spectral_norm
from ..models.sdxl import SDXLUNet, ddpm_alphas_cumprod


def apply_scaled_spectral_norm(module, iters=200):
    """Frozen-gain spectral norm on every trainable conv of ``module`` with ``iters`` power steps at
    set-up and one per forward in every mode (sd_guidance.py:51-89); ``algorithms.spectral`` does it."""
    return apply_spectral_norm(module, iters, update="always", types=(nn.Conv2d,))


def make_head(ch=1280, spatial=32):
    """Stride-2 convs down to 4x4, a 4x4/stride-4 conv, a 1x1 conv (three stride-2 convs for the
    32x32 bottleneck of 1024-pixel images, as the reference head)."""
    layers, s = [], spatial
    while s > 4:
        layers += [nn.Conv2d(ch, ch, 4, 2, 1), nn.GroupNorm(32, ch), nn.SiLU()]
        s //= 2
    layers += [nn.Conv2d(ch, ch, 4, 4, 0), nn.GroupNorm(32, ch), nn.SiLU(), nn.Conv2d(ch, 1, 1)]
    return nn.Sequential(*layers)


@dataclass
class SDXLDMADConfig:
    resolution: int = 1024
    latent: int = 128
    num_denoising_step: int = 4
    denoising_timestep: int = 1000
    critic_max_timestep: int = 1000
    teacher_gap_route: bool = True
    gap_tau: float = 0.5
    critic_spectral_norm: bool = True
    sn_iters: int = 200
    generator_lr: float = 5e-7
    guidance_lr: float = 5e-7
    # defaults of the reference's SDXL launcher (experiments/sdxl/train_common.sh)
    betas: tuple = (0.0, 0.99)
    teacher_loss_weight: float = 5e-3
    real_loss_weight: float = 5e-3
    critic_loss_weight: float = 1e-2
    generator_spectral_norm: bool = True  # frozen-gain SN on the generator's encoder + mid-block convs
    warmup_steps: int = 500  # learning rate ramps linearly from 0 over these steps (constant afterwards)
    # one-step generator (the reference's 1-step runs): pure noise in at this timestep, no backward
    # simulation; None = the multi-step generator of num_denoising_step steps
    conditioning_timestep: int | None = None
    backward_simulation: bool = True
    gradient_checkpointing: bool = True
    unet_kwargs: dict | None = None
    batch_size: int = 4  # per GPU (config 4)
    # the reference trainer's optimiser settings (train_sd.py:130-137, :246, :249-257): AdamW weight decay,
    # gradient clipping of both nets, and a generator EMA with a half-life of ema_kimg thousand images
    # (ramped up to ema_rampup x the images seen), exported as pytorch_model_ema.bin
    weight_decay: float = 0.01
    max_grad_norm: float = 10.0
    ema_kimg: float = 1000.0
    ema_rampup: float = 0.05
    # data-parallel optimiser: "sharded" = fp32 state sharded over the ranks, one fused reduce-scatter /
    # AdamW / all-gather kernel per step; "nccl" = NCCL all-reduce of the gradients, then torch's AdamW
    # on every rank (the library path, as the reference's accelerate DDP + AdamW)
    dp_optimizer: str = "sharded"


class SDXLDMAD:
    def __init__(self, cfg: SDXLDMADConfig = SDXLDMADConfig(), device="cuda", dtype=torch.bfloat16, seed=0):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        torch.manual_seed(seed)
        teacher = SDXLUNet(**(cfg.unet_kwargs or {}))
        self.generator = teacher
        self.critic = copy.deepcopy(teacher)
        self.critic.up_blocks = nn.ModuleList()
        self.critic.conv_norm_out = self.critic.conv_out = None
        ch = teacher.channels[-1]
        spatial = cfg.latent >> (len(teacher.channels) - 1)
        self.head_real, self.head_teacher = make_head(ch, spatial), make_head(ch, spatial)
        for m in self.head_teacher.modules():
            if isinstance(m, nn.Conv2d):
                nn.init.kaiming_normal_(m.weight, nonlinearity="relu")
                nn.init.zeros_(m.bias)
        if cfg.critic_spectral_norm:
            for mod in (self.critic.down_blocks, self.critic.mid_block, self.head_real, self.head_teacher):
                apply_scaled_spectral_norm(mod, cfg.sn_iters)
        if cfg.generator_spectral_norm:  # sd_unified_model.py:53-60
            for mod in (self.generator.down_blocks, self.generator.mid_block):
                apply_scaled_spectral_norm(mod, cfg.sn_iters)
        for m in (self.generator, self.critic):
            m.gradient_checkpointing = cfg.gradient_checkpointing
            m.to(self.device, dtype)
        self.head_real.to(self.device)
        self.head_teacher.to(self.device)
        self.ac = ddpm_alphas_cumprod().to(self.device)
        step = cfg.denoising_timestep // cfg.num_denoising_step
        self.step_list = torch.arange(cfg.denoising_timestep - 1, 0, -step, device=self.device)
        self.interval = step
        self.gap_ema = torch.zeros(NUM_GAP_BANDS, device=self.device)
        self.gap_ready = torch.zeros(NUM_GAP_BANDS, device=self.device)
        cp = list(self.critic.parameters()) + list(self.head_real.parameters()) + list(self.head_teacher.parameters())
        gp = [p for p in self.generator.parameters() if p.requires_grad]
        cp = [p for p in cp if p.requires_grad]
        from ..parallel.dist import broadcast_module
        for m in (self.generator, self.critic, self.head_real, self.head_teacher):
            broadcast_module(m)
        self.gen_params, self.critic_params_all = gp, cp
        self.gen_ema = None  # fp32 EMA of the generator (the nccl path; the sharded optimiser holds its own)
        if cfg.dp_optimizer == "sharded":
            from ..parallel.zero import ShardedAdamW
            self.opt_g = ShardedAdamW(gp, lr=cfg.generator_lr, betas=cfg.betas, weight_decay=cfg.weight_decay,
                                      ema=True)
            self.opt_c = ShardedAdamW(cp, lr=cfg.guidance_lr, betas=cfg.betas, weight_decay=cfg.weight_decay)
            self.sync_g = self.sync_c = None
        elif cfg.dp_optimizer == "nccl":
            from ..parallel.dp import GradSync
            self.opt_g = torch.optim.AdamW(gp, lr=cfg.generator_lr, betas=cfg.betas, weight_decay=cfg.weight_decay,
                                           foreach=True)
            self.opt_c = torch.optim.AdamW(cp, lr=cfg.guidance_lr, betas=cfg.betas, weight_decay=cfg.weight_decay,
                                           foreach=True)
            self.sync_g, self.sync_c = GradSync(gp), GradSync(cp)
            self.gen_ema = [p.detach().float().clone() for p in gp]
        else:
            raise ValueError(f"unknown dp_optimizer {cfg.dp_optimizer!r}")
        self.step_count = 0
        self.time_ids = torch.tensor([[cfg.resolution, cfg.resolution, 0, 0, cfg.resolution, cfg.resolution]],
                                     device=self.device, dtype=torch.float32)

    # ------------------------------------------------------------------ DDPM helpers
    def add_noise(self, x, eps, t):
        a = self.ac[t].reshape(-1, 1, 1, 1)
        return (a.sqrt() * x.double() + (1 - a).sqrt() * eps.double()).float()

    def x0_from_eps(self, xt, eps, t):
        a = self.ac[t].reshape(-1, 1, 1, 1)
        return ((xt.double() - (1 - a).sqrt() * eps.double()) / a.sqrt()).float()

    def unet(self, net, x, t, ctx, pooled, bottleneck=False):
        ids = self.time_ids.repeat(x.shape[0], 1)
        return net(x.to(self.dtype), t, ctx.to(self.dtype), ids, pooled.to(self.dtype), return_bottleneck=bottleneck)

    def _synced_int(self, hi):
        s = torch.randint(0, hi, (1,), device=self.device)
        if dist.is_available() and dist.is_initialized():
            dist.broadcast(s, 0)
        return int(s.item())

    @torch.no_grad()
    def sample_backward(self, noise, ctx, pooled):
        B = noise.shape[0]
        sel = self._synced_int(self.cfg.num_denoising_step)
        x, img = noise, noise
        for c in self.step_list[:sel]:
            t = torch.full((B,), int(c), device=self.device, dtype=torch.long)
            eps = self.unet(self.generator, x, t, ctx, pooled).float()
            img = self.x0_from_eps(x, eps, t)
            x = self.add_noise(img, torch.randn_like(img), t - self.interval)
        return img, torch.full((B,), int(self.step_list[sel]), device=self.device, dtype=torch.long)

    # ------------------------------------------------------------------ critic
    def critic_logits(self, x, t, ctx, pooled):
        xt = self.add_noise(x, torch.randn_like(x), t)
        rep = self.unet(self.critic, xt, t, ctx, pooled, bottleneck=True).float()
        return self.head_real(rep).reshape(-1), self.head_teacher(rep).reshape(-1)

    def gap_weight(self, t):
        if not self.cfg.teacher_gap_route:
            return None
        n_reach = min(NUM_GAP_BANDS, max(1, self.cfg.critic_max_timestep // 100 + 1))
        if float(self.gap_ready.sum()) < max(2, (n_reach + 1) // 2):
            return None
        center = float(self.gap_ema[self.gap_ready > 0].median())
        return torch.sigmoid((center - self.gap_ema[(t // 100).clamp(0, 9)]) / self.cfg.gap_tau)

    @torch.no_grad()
    def update_gap(self, dT, dQ, t):
        b = (t // 100).clamp(0, 9)
        s = torch.zeros(4, NUM_GAP_BANDS, device=self.device)
        s[0].scatter_add_(0, b, dT.float())
        s[1].scatter_add_(0, b, torch.ones_like(dT, dtype=torch.float32))
        s[2].scatter_add_(0, b, dQ.float())
        s[3].scatter_add_(0, b, torch.ones_like(dQ, dtype=torch.float32))
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(s)
        valid = (s[1] > 0) & (s[3] > 0)
        now = s[0] / s[1].clamp(min=1) - s[2] / s[3].clamp(min=1)
        upd = torch.where(valid & (self.gap_ready > 0), 0.99 * self.gap_ema + 0.01 * now, now)
        self.gap_ema.copy_(torch.where(valid, upd, self.gap_ema))
        self.gap_ready.copy_(torch.where(valid, torch.ones_like(self.gap_ready), self.gap_ready))

    def _critic_params(self):
        return list(self.critic.parameters()) + list(self.head_real.parameters()) + list(self.head_teacher.parameters())

    # ------------------------------------------------------------------ iteration
    def train_step(self, batch):
        """batch: noise / real / teacher latents [B, 4, 128, 128], ctx [B, 77, 2048], pooled [B, 1280]."""
        cfg = self.cfg
        noise, ctx, pooled = batch["noise"], batch["ctx"], batch["pooled"]
        B = noise.shape[0]
        self._apply_warmup()
        with torch.no_grad():
            if cfg.conditioning_timestep is not None:  # one-step generator: pure noise at a fixed timestep
                t = torch.full((B,), cfg.conditioning_timestep, device=self.device, dtype=torch.long)
                noisy = noise.clone()
            else:
                if cfg.backward_simulation:
                    clean, t = self.sample_backward(torch.randn_like(noise), ctx, pooled)
                else:
                    t = self.step_list[torch.randint(0, cfg.num_denoising_step, (B,), device=self.device)]
                    clean = batch["teacher"]
                noisy = self.add_noise(clean, noise, t)
                pure = t == cfg.denoising_timestep - 1
                noisy[pure] = noise[pure]
        self.generator.train()
        eps = self.unet(self.generator, noisy, t, ctx, pooled).float()
        G = self.x0_from_eps(noisy, eps, t)
        for p in self._critic_params():
            p.requires_grad_(False)
        tc = torch.randint(0, cfg.critic_max_timestep, (B,), device=self.device)
        dr, dt = self.critic_logits(G, tc, ctx, pooled)
        w = self.gap_weight(tc)
        tl = (-dt).mean() if w is None else (-dt * w).sum() / w.sum().clamp(min=1.0) + (-dt).sum() * 0.0
        loss_g = cfg.teacher_loss_weight * tl + cfg.real_loss_weight * (-dr).mean()
        loss_g.backward()
        decay = self.ema_decay(B)
        if self.sync_g is not None:
            self.sync_g.sync()
            torch.nn.utils.clip_grad_norm_(self.gen_params, cfg.max_grad_norm)
            self.opt_g.step()
            with torch.no_grad():
                torch._foreach_lerp_(self.gen_ema, [p.detach().float() for p in self.gen_params], 1.0 - decay)
        else:
            self.opt_g.step(ema_beta=decay, max_grad_norm=cfg.max_grad_norm)
        self.opt_g.zero_grad(set_to_none=True)
        for p in self._critic_params():
            p.requires_grad_(True)
        tc = torch.randint(0, cfg.critic_max_timestep, (B,), device=self.device)
        dR_T, _ = self.critic_logits(batch["real"], tc, ctx, pooled)
        dR_G, dQ_G = self.critic_logits(G.detach(), tc, ctx, pooled)
        dR_Q, dQ_Q = self.critic_logits(batch["teacher"], tc, ctx, pooled)
        loss_c = F.softplus(-dR_T).mean() + F.softplus(dR_G).mean() + F.softplus(-dQ_Q).mean() + F.softplus(dQ_G).mean()
        self.update_gap(dR_T.detach(), dR_Q.detach(), tc)
        (cfg.critic_loss_weight * loss_c).backward()
        if self.sync_c is not None:
            self.sync_c.sync()
            torch.nn.utils.clip_grad_norm_(self.critic_params_all, cfg.max_grad_norm)
            self.opt_c.step()
        else:
            self.opt_c.step(max_grad_norm=cfg.max_grad_norm)
        self.opt_c.zero_grad(set_to_none=True)
        self.step_count += 1
        return {"generator_loss": loss_g.detach(), "critic_loss": loss_c.detach()}

    def _apply_warmup(self):
        """Learning rates of this step: linear from 0 over warmup_steps, then constant (the reference's
        constant_with_warmup schedule, stepped after every optimiser step)."""
        w = self.cfg.warmup_steps
        done = getattr(self.opt_g, "step_count", self.step_count)
        f = 1.0 if w <= 0 else min(1.0, done / w)
        for opt, base in ((self.opt_g, self.cfg.generator_lr), (self.opt_c, self.cfg.guidance_lr)):
            if isinstance(opt, torch.optim.Optimizer):
                for g in opt.param_groups:
                    g["lr"] = base * f
            else:  # the sharded optimiser keeps one learning rate
                opt.lr = base * f

    # ------------------------------------------------------------------ generator EMA
    def ema_decay(self, batch: int) -> float:
        """Per-step EMA decay: half-life ema_kimg thousand images, at most ema_rampup x the images seen."""
        from ..parallel.dist import get_world_size
        total = batch * get_world_size()
        done = getattr(self.opt_g, "step_count", self.step_count)  # the sharded optimiser checkpoints its count
        nimg = (done + 1) * total
        half = self.cfg.ema_kimg * 1000
        if self.cfg.ema_rampup > 0:
            half = min(half, nimg * self.cfg.ema_rampup)
        return 0.5 ** (total / max(half, 1e-8))

    def ema_params(self) -> list:
        """The generator EMA, one full tensor per trainable generator parameter."""
        return self.opt_g.full_ema() if self.gen_ema is None else self.gen_ema

    def ema_state_dict(self) -> dict:
        """The generator's state dict with the EMA in place of its trainable weights."""
        sd = {k: v.detach().clone() for k, v in self.generator.state_dict().items()}
        names = {id(p): n for n, p in self.generator.named_parameters()}
        for p, e in zip(self.gen_params, self.ema_params()):
            sd[names[id(p)]] = e.detach().to("cpu", torch.float32).reshape(p.shape).clone()
        return sd

    def export_emas(self, out_dir: str):
        """``pytorch_model_ema.bin`` of a checkpoint, as the reference's trainer writes it (train_sd.py:209)."""
        import os

        os.makedirs(out_dir, exist_ok=True)
        torch.save({k: v.cpu() for k, v in self.ema_state_dict().items()}, os.path.join(out_dir, "pytorch_model_ema.bin"))

    def ema_state(self):
        """Checkpoint state of the EMA kept outside the optimiser (the nccl path)."""
        return None if self.gen_ema is None else {"gen_ema": [e.cpu() for e in self.gen_ema],
                                                  "step_count": self.step_count}

    def load_ema_state(self, st):
        if st is not None and self.gen_ema is not None:
            for d, v in zip(self.gen_ema, st["gen_ema"]):
                d.copy_(v.to(d.device))
        if st is not None:
            self.step_count = int(st.get("step_count", self.step_count))
