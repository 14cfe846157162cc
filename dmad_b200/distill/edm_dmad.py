"""DMAD for the EDM image generator (one-step student from sigma = 80), BASELINE config 1.

Parity with train/image/main/edm/edm_guidance.py and edm_unified_model.py / train_edm.py:
* critic = copy of the teacher U-Net with the decoder removed; two conv heads on the bottleneck
  (conv s2 -> GroupNorm -> SiLU ... -> 1x1 conv to one logit; adapted to the bottleneck size);
* frozen-gain spectral norm on every encoder / head conv (:54-80), optional on the generator encoder;
* critic noise: one shared level per sample, a uniform index into the 1000-level Karras grid (capped by
  ``critic_max_timestep``), or a lognormal sigma (config 1); optional clean critic;
* gap routing: bands = Karras index // 100, all-reduced sums, engaged when half of the reachable bands
  are measured, weighted-mean normalisation (:154-209);
* critic loss softplus BCE on both heads (+ optional R1 on T and Q, :211-267);
* one iteration = generator update (teacher / real loss weights) then critic update on the same batch,
  and the kimg half-life EMAs of the generator (train_edm.py:155-212).
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..algorithms.dmad import NUM_GAP_BANDS
from ..algorithms.ema import kimg_halflife_beta
from ..algorithms.spectral import attach_spectral_norm
from ..models.edm import EDMPrecond, config1_unet, load_edm_teacher


def get_sigmas_karras(n, sigma_min, sigma_max, rho=7.0):
    ramp = torch.linspace(0, 1, n)
    a, b = sigma_max ** (1 / rho), sigma_min ** (1 / rho)
    return (a + ramp * (b - a)) ** rho


def sn_wrap(module, power_iters=30):
    """Frozen-gain spectral norm on one Linear / Conv layer (gain fixed at its initial sigma_max,
    edm_guidance.py:54-80); the normalisation itself is ``algorithms.spectral``."""
    return int(attach_spectral_norm(module, power_iters))


def make_binary_head(channels, spatial):
    """Bottleneck [N, C, S, S] -> one logit: stride-2 convs down to 4x4, a 4x4/stride-4 conv, a 1x1 conv."""
    layers = []
    s = spatial
    while s > 4:
        layers += [nn.Conv2d(channels, channels, 4, stride=2, padding=1), nn.GroupNorm(32, channels), nn.SiLU()]
        s //= 2
    layers += [nn.Conv2d(channels, channels, 4, stride=4, padding=0), nn.GroupNorm(32, channels), nn.SiLU(),
               nn.Conv2d(channels, 1, 1)]
    return nn.Sequential(*layers)


@dataclass
class EDMDMADConfig:
    """Defaults: the reference's gap-routing ImageNet-64 recipe (experiments/imagenet/train_common.sh with
    dmad_imagenet_gaproute.sh: generator spectral norm, critic spectral norm and gap routing, critic noise
    capped at index 500, loss weights 3e-3, learning rates 2e-6 with a 500-step warm-up, generator EMAs of
    1000, 8000 and 16000 kimg)."""
    resolution: int = 64
    label_dim: int = 1000
    batch_size: int = 4
    conditioning_sigma: float = 80.0
    sigma_min: float = 0.002
    sigma_max: float = 80.0
    rho: float = 7.0
    num_train_timesteps: int = 1000
    min_step_percent: float = 0.02
    max_step_percent: float = 0.98
    critic_max_timestep: int | None = 500
    critic_sigma: str = "karras"        # "karras" | "lognormal" (config 1: P_mean -1.2, P_std 1.2)
    p_mean: float = -1.2
    p_std: float = 1.2
    critic_clean: bool = False
    critic_spectral_norm: bool = True
    generator_spectral_norm: bool = True
    teacher_gap_route: bool = True
    gap_tau: float = 0.5
    r1_gamma: float = 0.0
    r1_batch_size: int = 16
    pretrained_critic: str = ""          # e.g. "vgg16_bn,tf_efficientnet_lite0": Projected-GAN feature critic
    model_id: str = ""                   # pretrained EDM teacher (.pkl release pickle, .pt / .safetensors)
    teacher_loss_weight: float = 3e-3
    real_loss_weight: float = 3e-3
    generator_lr: float = 2e-6
    guidance_lr: float = 2e-6
    betas: tuple = (0.0, 0.99)
    max_grad_norm: float = 10.0
    ema_kimg: tuple = (1000.0, 8000.0, 16000.0)  # the first is the primary EMA
    ema_rampup: float = 0.05
    warmup_steps: int = 500  # learning rates ramp linearly from 0 over these steps (constant afterwards)


class EDMCritic(nn.Module):
    def __init__(self, cfg: EDMDMADConfig, teacher: EDMPrecond):
        super().__init__()
        self.cfg = cfg
        self.pg = None
        if cfg.pretrained_critic:
            # frozen feature networks + multi-scale heads instead of the teacher-encoder critic
            # (edm_guidance.py:87-91); no noise-level input
            from ..models.pg_critic import PGTwoHeadCritic

            self.pg = PGTwoHeadCritic([b for b in cfg.pretrained_critic.split(",") if b], c_dim=cfg.label_dim)
        else:
            self.fake_unet = copy.deepcopy(teacher)
            unet = self.fake_unet.model
            unet.dec, unet.out_norm, unet.out_conv = None, None, None
            c = unet.bottleneck_channels
            spatial = cfg.resolution >> (len([k for k in unet.enc.keys() if k.endswith("_down")]))
            self.head_real = make_binary_head(c, spatial)
            self.head_teacher = make_binary_head(c, spatial)
            if cfg.critic_spectral_norm:
                for m in list(unet.enc.modules()) + list(self.head_real.modules()) + list(self.head_teacher.modules()):
                    if isinstance(m, nn.Conv2d):
                        sn_wrap(m)
        self.register_buffer("karras", torch.flip(get_sigmas_karras(cfg.num_train_timesteps, cfg.sigma_min,
                                                                    cfg.sigma_max, cfg.rho), dims=[0]))
        self.register_buffer("gap_ema", torch.zeros(NUM_GAP_BANDS))
        self.register_buffer("gap_ready", torch.zeros(NUM_GAP_BANDS))
        self.min_step = int(cfg.min_step_percent * cfg.num_train_timesteps)
        self.max_step = int(cfg.max_step_percent * cfg.num_train_timesteps)

    def sample_timesteps(self, n, device):
        lo = max(0, min(self.min_step, self.cfg.num_train_timesteps - 1))
        hi = max(lo, min(self.max_step, self.cfg.num_train_timesteps - 1))
        if self.cfg.critic_max_timestep is not None:
            hi = max(lo, min(hi, self.cfg.critic_max_timestep))
        return torch.randint(lo, hi + 1, (n,), device=device)

    def draw_sigma(self, n, device):
        """(index into the Karras grid, sigma) per sample."""
        if self.cfg.critic_sigma == "lognormal":
            sig = torch.exp(torch.randn(n, device=device) * self.cfg.p_std + self.cfg.p_mean)
            idx = torch.searchsorted(self.karras, sig.contiguous()).clamp(0, self.cfg.num_train_timesteps - 1)
            return idx, sig
        idx = self.sample_timesteps(n, device)
        return idx, self.karras[idx]

    def set_trainable(self, flag: bool):
        """Critic parameters on / off for autograd; the feature networks of the pretrained critic stay frozen."""
        self.requires_grad_(flag)
        if self.pg is not None:
            self.pg.features.requires_grad_(False)

    def logits(self, x, sigma, labels):
        """(d_real, d_teacher): [N] each, or [N, K] per-pixel logits with the pretrained critic."""
        if self.pg is not None:
            return self.pg(x, labels)
        rep = self.fake_unet(x, sigma, labels, return_bottleneck=True).float()
        return self.head_real(rep).reshape(-1), self.head_teacher(rep).reshape(-1)

    @staticmethod
    def _per_sample(d):
        return d if d.dim() == 1 else d.float().mean(1)

    @torch.no_grad()
    def update_gap(self, d_T, d_Q, idx_T, idx_Q):
        bt, bq = (idx_T // 100).clamp(0, 9), (idx_Q // 100).clamp(0, 9)
        dev = d_T.device
        s = torch.zeros(4, NUM_GAP_BANDS, device=dev)
        s[0].scatter_add_(0, bt, d_T.float())
        s[1].scatter_add_(0, bt, torch.ones_like(d_T, dtype=torch.float32))
        s[2].scatter_add_(0, bq, d_Q.float())
        s[3].scatter_add_(0, bq, torch.ones_like(d_Q, dtype=torch.float32))
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(s)
        valid = (s[1] > 0) & (s[3] > 0)
        now = s[0] / s[1].clamp(min=1) - s[2] / s[3].clamp(min=1)
        upd = torch.where(valid & (self.gap_ready > 0), 0.99 * self.gap_ema + 0.01 * now, now)
        self.gap_ema.copy_(torch.where(valid, upd, self.gap_ema))
        self.gap_ready.copy_(torch.where(valid, torch.ones_like(self.gap_ready), self.gap_ready))

    def gap_weight(self, idx):
        if not self.cfg.teacher_gap_route:
            return None
        tmax = self.cfg.critic_max_timestep
        n_reach = 10 if tmax is None else min(10, max(1, int(tmax) // 100 + 1))
        if float(self.gap_ready.sum()) < max(2, (n_reach + 1) // 2):
            return None
        center = float(self.gap_ema[self.gap_ready > 0].median())
        return torch.sigmoid((center - self.gap_ema[(idx // 100).clamp(0, 9)]) / self.cfg.gap_tau)

    def generator_loss(self, image, labels):
        B = image.shape[0]
        if self.cfg.critic_clean:
            idx = torch.zeros(B, dtype=torch.long, device=image.device)
            sig = self.karras[0].expand(B)
            noisy = image
        else:
            idx, sig = self.draw_sigma(B, image.device)
            noisy = image + sig.reshape(-1, 1, 1, 1) * torch.randn_like(image)
        d_r, d_t = self.logits(noisy, sig, labels)
        w = self.gap_weight(idx)
        x = -d_t
        if w is not None and x.dim() == 2:  # per-pixel logits: the sample's weight on each of its logits
            w = w[:, None].expand_as(x)
        tl = x.mean() if w is None else (x * w).sum() / w.sum().clamp(min=1.0) + x.sum() * 0.0
        return {"gen_teacher_loss": tl, "gen_real_loss": (-d_r).mean()}

    def r1(self, xT, xQ, sT, sQ, lT, lQ):
        k = max(1, min(xT.shape[0], self.cfg.r1_batch_size))
        a = xT[:k].detach().requires_grad_(True)
        dr, _ = self.logits(a, sT[:k], lT[:k])
        g1 = torch.autograd.grad(self._per_sample(dr).sum(), a, create_graph=True)[0]
        b = xQ[:k].detach().requires_grad_(True)
        _, dq = self.logits(b, sQ[:k], lQ[:k])
        g2 = torch.autograd.grad(self._per_sample(dq).sum(), b, create_graph=True)[0]
        return 0.5 * (g1.pow(2).flatten(1).sum(1).mean() + g2.pow(2).flatten(1).sum(1).mean())

    def critic_loss(self, fake, real, fake_l, real_l, teacher, teacher_l):
        B = fake.shape[0]
        idx, sig = self.draw_sigma(B, fake.device)
        real, fake, teacher = real.detach(), fake.detach(), teacher.detach()
        if self.cfg.critic_clean:
            sig = self.karras[0].expand(B)
            xT, xG, xQ = real, fake, teacher
        else:
            s4 = sig.reshape(-1, 1, 1, 1)
            xT, xG, xQ = real + s4 * torch.randn_like(real), fake + s4 * torch.randn_like(fake), \
                teacher + s4 * torch.randn_like(teacher)
        if self.pg is not None:
            # one forward per image set, so the heads' BatchNorms see the batches the generator step sees
            parts = [self.logits(x, sig, lab) for x, lab in ((xT, real_l), (xG, fake_l), (xQ, teacher_l))]
            d_r, d_t = torch.cat([p[0] for p in parts]), torch.cat([p[1] for p in parts])
        else:
            d_r, d_t = self.logits(torch.cat([xT, xG, xQ]), torch.cat([sig, sig, sig]),
                                   torch.cat([real_l, fake_l, teacher_l]))
        dR_T, dR_G, dR_Q = d_r[:B], d_r[B:2 * B], d_r[2 * B:]
        dQ_G, dQ_Q = d_t[B:2 * B], d_t[2 * B:]
        if self.cfg.teacher_gap_route:
            self.update_gap(self._per_sample(dR_T.detach()), self._per_sample(dR_Q.detach()), idx, idx)
        loss = F.softplus(-dR_T).mean() + F.softplus(dR_G).mean() + F.softplus(-dQ_Q).mean() + F.softplus(dQ_G).mean()
        log = {"critic_acc_t": (dR_T > 0).float().mean().detach(), "critic_acc_q": (dQ_Q > 0).float().mean().detach(),
               "critic_acc_g": (0.5 * ((dR_G < 0).float().mean() + (dQ_G < 0).float().mean())).detach()}
        if self.cfg.r1_gamma > 0:
            r1 = self.r1(xT, xQ, sig, sig, real_l, teacher_l)
            loss = loss + 0.5 * self.cfg.r1_gamma * r1
            log["r1"] = r1.detach()
        return loss, log


class EDMDMAD:
    """Generator (one step from sigma = 80) + two-head critic, trained 1:1 per iteration."""

    def __init__(self, cfg: EDMDMADConfig = EDMDMADConfig(), teacher: EDMPrecond | None = None, device="cpu"):
        self.cfg, self.device = cfg, torch.device(device)
        if teacher is None:
            teacher = config1_unet(cfg.label_dim)
            if cfg.model_id:  # it initialises the generator and the critic backbone (edm_unified_model.py:13-30)
                load_edm_teacher(teacher, cfg.model_id)
        self.critic = EDMCritic(cfg, teacher).to(self.device)
        self.generator = copy.deepcopy(teacher).to(self.device)
        if cfg.generator_spectral_norm:
            for m in self.generator.model.enc.modules():
                if isinstance(m, nn.Conv2d):
                    sn_wrap(m)
        self.opt_g = torch.optim.AdamW(self.generator.parameters(), lr=cfg.generator_lr, betas=cfg.betas)
        self.opt_c = torch.optim.AdamW([p for p in self.critic.parameters() if p.requires_grad], lr=cfg.guidance_lr,
                                       betas=cfg.betas)
        self.emas = {k: copy.deepcopy(self.generator).requires_grad_(False) for k in cfg.ema_kimg}
        self.step_count = 0
        self.eye = torch.eye(cfg.label_dim, device=self.device)

    def ema_state(self) -> dict:
        """Trainer state outside the modules and optimisers: the step count (learning-rate warm-up, EMA ramp-up)."""
        return {"step_count": self.step_count}

    def load_ema_state(self, st):
        self.step_count = int(st.get("step_count", self.step_count))

    def ema_files(self) -> dict:
        """{file name: EMA generator} in the reference's checkpoint naming (train_edm.py:106-124): the
        first of ``ema_kimg`` is the primary ``pytorch_model_ema.bin``, every other one
        ``pytorch_model_ema_<int(kimg)>.bin``."""
        out = {}
        for i, (kimg, ema) in enumerate(self.emas.items()):
            out["pytorch_model_ema.bin" if i == 0 else f"pytorch_model_ema_{int(kimg)}.bin"] = ema
        return out

    def export_emas(self, out_dir: str):
        """Writes the generator EMAs of a checkpoint as plain EDMPrecond state dicts (spectral norm, if
        any, folded into the weights), loadable by the reference's networks and by ``tools.edm_eval_folder``."""
        import os

        from ..algorithms.spectral import fold_spectral_norm

        os.makedirs(out_dir, exist_ok=True)
        for name, ema in self.ema_files().items():
            net = copy.deepcopy(ema).cpu().eval()
            with torch.no_grad():
                fold_spectral_norm(net)
            torch.save(net.state_dict(), os.path.join(out_dir, name))

    def synthetic_batch(self, gen: torch.Generator | None = None):
        """Config-1 inputs: images U[-1, 1], labels U{0..999}; teacher samples drawn the same way."""
        c, B, r = self.cfg, self.cfg.batch_size, self.cfg.resolution
        real = torch.rand(B, 3, r, r, generator=gen) * 2 - 1
        teach = torch.rand(B, 3, r, r, generator=gen) * 2 - 1
        lr = torch.randint(0, c.label_dim, (B,), generator=gen)
        lt = torch.randint(0, c.label_dim, (B,), generator=gen)
        lab = torch.randint(0, c.label_dim, (B,), generator=gen)
        noise = torch.randn(B, 3, r, r, generator=gen) * c.conditioning_sigma
        d = self.device
        return {"real_image": real.to(d), "real_label": self.eye[lr.to(d)], "second_real_image": teach.to(d),
                "second_real_label": self.eye[lt.to(d)], "noise": noise.to(d), "labels": self.eye[lab.to(d)]}

    def train_step(self, batch):
        c = self.cfg
        f = 1.0 if c.warmup_steps <= 0 else min(1.0, self.step_count / c.warmup_steps)
        for opt, base in ((self.opt_g, c.generator_lr), (self.opt_c, c.guidance_lr)):
            for g in opt.param_groups:  # constant_with_warmup, stepped after every optimiser step
                g["lr"] = base * f
        B = batch["noise"].shape[0]
        sigma = torch.full((B,), c.conditioning_sigma, device=self.device)
        self.generator.train()
        self.critic.train()
        gen = self.generator(batch["noise"], sigma, batch["labels"])
        self.critic.set_trainable(False)
        gl = self.critic.generator_loss(gen, batch["labels"])
        self.critic.set_trainable(True)
        loss_g = gl["gen_teacher_loss"] * c.teacher_loss_weight + gl["gen_real_loss"] * c.real_loss_weight
        loss_g.backward()
        gnorm = torch.nn.utils.clip_grad_norm_(self.generator.parameters(), c.max_grad_norm)
        self.opt_g.step()
        self.opt_g.zero_grad()
        self.opt_c.zero_grad()
        nimg = (self.step_count + 1) * B
        for kimg, ema in self.emas.items():
            beta = kimg_halflife_beta(B, nimg, kimg, c.ema_rampup)
            with torch.no_grad():
                for pe, p in zip(ema.parameters(), self.generator.parameters()):
                    pe.mul_(beta).add_(p.detach(), alpha=1 - beta)
        loss_c, log = self.critic.critic_loss(gen.detach(), batch["real_image"], batch["labels"], batch["real_label"],
                                              batch["second_real_image"], batch["second_real_label"])
        loss_c.backward()
        cnorm = torch.nn.utils.clip_grad_norm_([p for p in self.critic.parameters() if p.requires_grad], c.max_grad_norm)
        self.opt_c.step()
        self.opt_c.zero_grad()
        self.opt_g.zero_grad()
        self.step_count += 1
        out = {"generator_loss": float(loss_g.detach()), "critic_loss": float(loss_c.detach()), "generator_grad_norm": float(gnorm),
               "guidance_grad_norm": float(cnorm)}
        out.update({k: float(v) for k, v in log.items()})
        return out
