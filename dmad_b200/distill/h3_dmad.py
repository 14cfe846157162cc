"""DMAD distillation of the H3-shaped audio-video DiT.

Parity with train/h3/lightx2v_train/trainers/dmd/minimax_h3_dmad_trainer.py and its rollout base
(minimax_h3_trainer.py, trainers/dmd/trainer.py):
* per iteration one student stage, then ``fake_update_ratio`` critic stages (trainer.py:129-145);
* rollout length ``end_step_idx`` drawn uniformly in [0, num_inference_steps) and broadcast from rank 0;
  ``end_step_idx + 1`` student evaluations, only the last with grad, DMD2 re-noise between them; the
  levels are a running minimum of U[min, max] draws, flow-shifted per modality (video 12, audio 2);
  velocity is data-ward: x0 = x_t + sigma v (minimax_h3_trainer.py:105-164);
* critic = the fake model truncated after ``feature_block`` (the later blocks never run), tokens
  normalised by a non-affine RMSNorm, two Linear-SiLU-Linear heads, logits pooled as the mean of the
  audio-token mean and the video-token mean (:262-295);
* G / T / Q share one critic noise level (U[min, max] then shifted); critic loss softplus BCE, student
  loss -d_real(G) - (w/E_w) d_teacher(G) with the per-rank, bias-corrected gap EMA in 10 CDF-decile
  bands of the pre-shift uniform (:305-378);
* critic frozen through the student backward; head gradients all-reduced (AVG) before the head step;
* two power-EMA banks of the student's trainable weights, gamma 6.94 and 16.97 (:458-480);
* full-critic mode freezes the refiner, embedders and blocks[:k] (:160-180).
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass, field
from pathlib import Path

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..algorithms import CriticHeads, GapRouter, PowerEMA, critic_bce_loss, generator_linear_loss
from ..algorithms.dmad import NUM_GAP_BANDS
from ..inference.h3 import H3Geometry, build_packed_sequence, build_row_timesteps, latent_shape_of, shift_sigma
from ..models.h3 import H3Config, H3Model
from ..ops.optim import FusedAdamW
from ..parallel.dist import broadcast_module, get_world_size
from ..parallel.dp import GradSync


@dataclass
class H3DMADConfig:
    model: H3Config = field(default_factory=H3Config)
    height: int = 768
    width: int = 1344
    num_frames: int = 124
    num_inference_steps: int = 4
    fake_update_ratio: int = 1
    renoise_sigma_min: float = 0.02
    renoise_sigma_max: float = 0.98
    video_shift: float = 12.0
    audio_shift: float = 2.0
    feature_block: int = -1
    gap_tau: float = 2.0
    ema_gammas: tuple = (6.94, 16.97)
    student_lora_rank: int = 128
    fake_train_type: str = "lora"     # "lora" | "full"
    critic_freeze_blocks: int = 25
    lr: float = 4e-5
    fake_lr: float = 4e-5
    betas: tuple = (0.0, 0.99)
    weight_decay: float = 0.01
    eps: float = 1e-8
    head_lr: float = 4e-5
    head_wd: float = 0.01
    gradient_checkpointing: bool = True
    text_tokens: int = 256
    model_dir: str | None = None      # H3 release folder: transformer/config.json sets ``model``, shards load
    # shard the block weights over the ranks (FSDP-style, the reference's fully_shard per block,
    # train/h3/lightx2v_train/runtime/fsdp.py:35-85): the frozen bases of the LoRA student and critic,
    # and in full-critic mode the critic's trainable blocks (gathered one block ahead, gradients
    # reduce-scattered per block, AdamW on the shards); needs gradient_checkpointing
    shard_weights: bool = False


class SyntheticH3Pool:
    """N(0,1) stand-in for the real-latent pool with the shapes of the configured tier."""

    def __init__(self, shape, text_tokens, text_dim, geometry: H3Geometry, seed=0):
        self.shape, self.nt, self.text_dim, self.geo = shape, text_tokens, text_dim, geometry
        self.g = torch.Generator().manual_seed(seed)

    def draw_condition(self):
        return {"prompt_embeds": torch.randn(1, self.nt, self.text_dim, generator=self.g),
                "text_token_tags": torch.ones(self.nt, dtype=torch.long)}

    def draw(self, device, dtype=torch.float32):
        s, geo = self.shape, self.geo
        v = torch.randn(geo.video_latent_channels, s["latent_frames"], s["latent_height"], s["latent_width"],
                        generator=self.g)
        a = torch.randn(2, s["audio_latents"], geo.audio_latent_channels, generator=self.g)
        tv = torch.randn(s["video_tokens"], generator=self.g)
        ta = torch.randn(s["audio_tokens"], generator=self.g)
        return v.to(device, dtype), a.to(device, dtype), tv.to(device, dtype), ta.to(device, dtype), \
            self.draw_condition()


class H3DMAD:
    def __init__(self, cfg: H3DMADConfig, device, pool=None, dtype=torch.bfloat16, seed=0):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.geo = H3Geometry()
        if cfg.model_dir:
            # the pretrained transformer (reference: model_zoo/minimax_h3_t2av.py:15-60 loads it from the
            # Diffusers folder); the network's shape comes from its config.json
            from ..inference.h3 import config_from_transformer_dir
            cfg.model = config_from_transformer_dir(cfg.model_dir)
            if (Path(cfg.model_dir) / "vae" / "config.json").is_file():
                self.geo = H3Geometry.from_model_dir(cfg.model_dir)
        self.shape = latent_shape_of(cfg.height, cfg.width, cfg.num_frames, self.geo)
        torch.manual_seed(seed)
        if self.device.type == "cuda":
            # built on the device in the compute dtype: two 33B nets are 132 GB in bf16, far beyond what
            # fp32 host copies per rank could hold
            prev = torch.get_default_dtype()
            torch.set_default_dtype(dtype)
            try:
                with torch.device(self.device):
                    base = H3Model(cfg.model)
            finally:
                torch.set_default_dtype(prev)
        else:
            base = H3Model(cfg.model)
        if cfg.model_dir:
            from ..inference.h3 import load_transformer_weights
            load_transformer_weights(base, cfg.model_dir)
        self.student = base
        self.fake = copy.deepcopy(base)
        self.student.enable_lora(cfg.student_lora_rank)
        if cfg.fake_train_type == "lora":
            self.fake.enable_lora(cfg.student_lora_rank)
        else:
            frozen = [self.fake.token_refiner, self.fake.proj_in, self.fake.audio_proj_in, self.fake.context_embedder,
                      self.fake.time_embedder] + list(self.fake.transformer_blocks[: cfg.critic_freeze_blocks])
            for m in frozen:
                m.requires_grad_(False)
        self.student.to(self.device, dtype)
        self.fake.to(self.device, dtype)
        if cfg.gradient_checkpointing:
            self.student.checkpoint_blocks = len(self.student.transformer_blocks)
            self.fake.checkpoint_blocks = len(self.fake.transformer_blocks)
        self.heads = CriticHeads(cfg.model.dim, rms_input=True).to(self.device, torch.float32)
        for m in (self.student, self.fake, self.heads):
            broadcast_module(m)
        self.fb = cfg.feature_block % len(self.fake.transformer_blocks)
        self.s_params = [p for p in self.student.parameters() if p.requires_grad]
        self.f_params = [p for p in self.fake.parameters() if p.requires_grad]
        self.sharded = []
        owned = set()
        if cfg.shard_weights:
            from ..parallel.fsdp import ShardedFrozenBlocks, ShardedTrainableBlocks
            if not cfg.gradient_checkpointing:
                raise ValueError("shard_weights needs gradient_checkpointing (the blocks are gathered per use)")
            self.sharded.append(ShardedFrozenBlocks(self.student.transformer_blocks))
            fblocks = list(self.fake.transformer_blocks)
            if cfg.fake_train_type == "lora":
                self.sharded.append(ShardedFrozenBlocks(fblocks))
            else:
                k = min(cfg.critic_freeze_blocks, len(fblocks))
                if k > 0:
                    self.sharded.append(ShardedFrozenBlocks(fblocks[:k]))
                if k < len(fblocks):
                    self.fake_fsdp = ShardedTrainableBlocks(fblocks[k:], lr=cfg.fake_lr, betas=cfg.betas, eps=cfg.eps,
                                                            weight_decay=cfg.weight_decay)
                    self.sharded.append(self.fake_fsdp)
                    owned = {id(p) for p in self.fake_fsdp.params}
        self.opt_s = FusedAdamW(self.s_params, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps, weight_decay=cfg.weight_decay)
        f_rest = [p for p in self.f_params if id(p) not in owned]
        self.opt_f = FusedAdamW(f_rest, lr=cfg.fake_lr, betas=cfg.betas, eps=cfg.eps, weight_decay=cfg.weight_decay)
        if owned:
            from ..parallel.fsdp import FSDPOptimizer
            self.opt_f = FSDPOptimizer(self.fake_fsdp, self.opt_f)
        # the heads' AdamW is the same multi-tensor kernel (fp32 parameters act as their own master copy)
        self.opt_h = FusedAdamW(list(self.heads.parameters()), lr=cfg.head_lr, betas=cfg.betas,
                                weight_decay=cfg.head_wd, eps=cfg.eps)
        self.sync_s, self.sync_f = GradSync(self.s_params), GradSync(f_rest)
        self.gap = GapRouter("local", tau=cfg.gap_tau, beta=0.99, min_ready=5, band_min_count=10).to(self.device)
        self.ema_banks = [PowerEMA(self.s_params, g) for g in cfg.ema_gammas]
        self.pool = pool or SyntheticH3Pool(self.shape, cfg.text_tokens, cfg.model.text_dim, self.geo, seed=seed)
        self._layout_cache = {}
        self.student_steps = 0

    # ------------------------------------------------------------------ helpers
    def layout(self, cond):
        tags = cond["text_token_tags"]
        key = int(tags.numel())
        if key not in self._layout_cache:
            s = self.shape
            self._layout_cache[key] = build_packed_sequence(tags, s["latent_frames"], s["latent_height"],
                                                            s["latent_width"], s["audio_latents"],
                                                            self.geo.patch_size).to(self.device)
        return self._layout_cache[key]

    def _synced_int(self, low, high):
        t = torch.randint(low, high, (1,), device=self.device)
        if dist.is_available() and dist.is_initialized():
            dist.broadcast(t, src=0)
        return int(t.item())

    def _uniform(self):
        return torch.empty((), device=self.device).uniform_(self.cfg.renoise_sigma_min, self.cfg.renoise_sigma_max)

    def velocity(self, model, x, sigmas, cond, lay, stop_after=None):
        ts, ti = build_row_timesteps(lay, sigmas[0], sigmas[1])
        return model(hidden_states=x[0], audio_hidden_states=x[1],
                     encoder_hidden_states=cond["prompt_embeds"].to(self.device, self.dtype),
                     timestep=ts.to(self.device), timestep_indices=ti.to(self.device), token_tags=lay.token_tags,
                     position_ids=lay.position_ids, video_indices=lay.video_indices, audio_indices=lay.audio_indices,
                     text_indices=lay.text_indices, stop_after_block=stop_after)

    def rollout_sigmas(self, end):
        base = torch.ones(end + 2, device=self.device)
        run = base[0]
        for i in range(1, end + 1):
            run = torch.minimum(self._uniform(), run)
            base[i] = run
        base[-1] = 0.0
        return shift_sigma(base, self.cfg.video_shift), shift_sigma(base, self.cfg.audio_shift)

    def back_simulation(self, cond, end, grad):
        lay = self.layout(cond)
        xt = (torch.randn(self.shape["video_tokens"], device=self.device),
              torch.randn(self.shape["audio_tokens"], device=self.device))
        vs, as_ = self.rollout_sigmas(end)
        self.student.train()
        x0 = None
        for k in range(end + 1):
            with torch.set_grad_enabled(grad and k == end):
                v = self.velocity(self.student, xt, (vs[k], as_[k]), cond, lay)
                x0 = (xt[0] + vs[k] * v[0].float(), xt[1] + as_[k] * v[1].float())
            if k == end:
                break
            with torch.no_grad():
                n = (torch.randn_like(x0[0]), torch.randn_like(x0[1]))
                xt = self.add_noise((x0[0].detach(), x0[1].detach()), n, (vs[k + 1], as_[k + 1]))
        return x0

    @staticmethod
    def add_noise(x, n, s):
        return ((1.0 - s[0]) * x[0].float() + s[0] * n[0], (1.0 - s[1]) * x[1].float() + s[1] * n[1])

    def critic_logits(self, x, sigmas, cond):
        lay = self.layout(cond)
        tok = self.velocity(self.fake, x, sigmas, cond, lay, stop_after=self.fb)
        ai, vi = lay.audio_indices, lay.video_indices
        d_r, d_t = self.heads(tok[:, torch.cat([ai, vi])].float())
        na = ai.numel()

        def pool(d):
            return ((d[:, :na].mean(dim=1) + d[:, na:].mean(dim=1)) / 2.0).squeeze(-1)

        return pool(d_r), pool(d_t)

    def sigma_band(self, video_sigma):
        sp, sh = float(video_sigma), self.cfg.video_shift
        u = sp / (sh - (sh - 1.0) * sp)
        return min(NUM_GAP_BANDS - 1, max(0, int(u * NUM_GAP_BANDS)))

    def pack_real(self, video, audio):
        _, ph, pw = self.geo.patch_size
        c, t, h, w = video.shape
        v = video.reshape(c, t, h // ph, ph, w // pw, pw).permute(1, 2, 4, 0, 3, 5)
        v = v.reshape(1, t * (h // ph) * (w // pw), c * ph * pw)
        a = audio.reshape(1, audio.shape[0] * audio.shape[1], audio.shape[2])
        if tuple(v.shape) != tuple(self.shape["video_tokens"]) or tuple(a.shape) != tuple(self.shape["audio_tokens"]):
            raise RuntimeError(f"real latent shape {tuple(v.shape)}/{tuple(a.shape)} != expected")
        return v, a

    def _freeze_critic(self, freeze):
        for p in self.f_params:
            p.requires_grad_(not freeze)
        self.heads.requires_grad_(not freeze)

    # ------------------------------------------------------------------ stages
    def student_stage(self):
        cond = self.pool.draw_condition()
        end = self._synced_int(0, self.cfg.num_inference_steps)
        G = self.back_simulation(cond, end, True)
        base = self._uniform()
        sig = (shift_sigma(base, self.cfg.video_shift), shift_sigma(base, self.cfg.audio_shift))
        xg = self.add_noise(G, (torch.randn_like(G[0]), torch.randn_like(G[1])), sig)
        self._freeze_critic(True)
        self.fake.eval()
        try:
            d_r, d_t = self.critic_logits(xg, sig, cond)
            w, E_w = self.gap.weights(torch.tensor([self.sigma_band(sig[0])]))
            wgt = (w / E_w).mean() if w is not None else 1.0
            loss = (-d_r).mean() + wgt * (-d_t).mean()
            loss.backward()
        finally:
            self._freeze_critic(False)
            self.fake.train()
        self.sync_s.sync()
        self.opt_s.step()
        self.opt_s.zero_grad()
        self.student_steps += 1
        for bank in self.ema_banks:
            bank.update()
        return {"loss": float(loss.detach()), "d_g": float(d_r.detach().mean()), "d_g_teacher": float(d_t.detach().mean()),
                "gap_w": float(wgt)}

    def critic_stage(self):
        rv, ra, tv, ta, cond = self.pool.draw(self.device)
        end = self._synced_int(0, self.cfg.num_inference_steps)
        with torch.no_grad():
            G = self.back_simulation(cond, end, False)
        base = self._uniform()
        sig = (shift_sigma(base, self.cfg.video_shift), shift_sigma(base, self.cfg.audio_shift))
        self.fake.train()
        real = self.pack_real(rv, ra)
        xg = self.add_noise((G[0].detach(), G[1].detach()), (torch.randn_like(G[0]), torch.randn_like(G[1])), sig)
        d_g_r, d_g_t = self.critic_logits(xg, sig, cond)
        (F.softplus(d_g_t) + F.softplus(d_g_r)).mean().backward()
        xT = self.add_noise(real, (torch.randn_like(real[0]), torch.randn_like(real[1])), sig)
        d_t, _ = self.critic_logits(xT, sig, cond)
        F.softplus(-d_t).mean().backward()
        xQ = self.add_noise((tv, ta), (torch.randn_like(tv), torch.randn_like(ta)), sig)
        d_q_r, d_q = self.critic_logits(xQ, sig, cond)
        F.softplus(-d_q).mean().backward()
        bce = critic_bce_loss(d_t.detach(), d_g_r.detach(), d_q.detach(), d_g_t.detach()).mean()
        self.gap.update_local(self.sigma_band(sig[0]), d_t, d_q_r)
        self.sync_f.sync()
        if get_world_size() > 1:
            for p in self.heads.parameters():
                if p.grad is not None:
                    dist.all_reduce(p.grad)
                    p.grad.div_(get_world_size())
        self.opt_h.step()
        self.opt_h.zero_grad()
        self.opt_f.step()
        self.opt_f.zero_grad()
        return {"gan_d": float(bce), "acc_t": float((d_t > 0).float().mean()), "acc_q": float((d_q > 0).float().mean()),
                "acc_g": float(0.5 * ((d_g_r < 0).float().mean() + (d_g_t < 0).float().mean()))}

    def train_iteration(self):
        out = {"student": self.student_stage()}
        for k in range(self.cfg.fake_update_ratio):
            out[f"critic{k}"] = self.critic_stage()
        return out

    # ------------------------------------------------------------------ checkpoint pieces
    @torch.no_grad()
    def export_loras(self, out_dir: str):
        """The checkpoint's LoRA files in the Diffusers layout: the live student
        (``pytorch_lora_weights.safetensors``), one directory per power-EMA bank (``ema_lora/``,
        ``ema2_lora/``) and the critic (``fake_lora/``) (minimax_h3_dmad_trainer.py:543-595)."""
        import os

        from ..lora import lora_pairs_from_model, save_lora_file

        os.makedirs(out_dir, exist_ok=True)
        r = self.cfg.student_lora_rank
        save_lora_file(os.path.join(out_dir, "pytorch_lora_weights.safetensors"),
                       lora_pairs_from_model(self.student, torch.bfloat16), r, r)
        for k, bank in enumerate(self.ema_banks):
            live = [p.detach().clone() for p in bank.params]
            for p, sh in zip(bank.params, bank.shadow):
                p.copy_(sh.to(p.dtype))
            d = os.path.join(out_dir, "ema_lora" if k == 0 else f"ema{k + 1}_lora")
            os.makedirs(d, exist_ok=True)
            save_lora_file(os.path.join(d, "pytorch_lora_weights.safetensors"),
                           lora_pairs_from_model(self.student, torch.bfloat16), r, r,
                           {"ema_gamma": str(bank.gamma), "ema_t": str(bank.t)})
            for p, v in zip(bank.params, live):
                p.copy_(v)
        if self.cfg.fake_train_type == "lora":
            d = os.path.join(out_dir, "fake_lora")
            os.makedirs(d, exist_ok=True)
            save_lora_file(os.path.join(d, "pytorch_lora_weights.safetensors"),
                           lora_pairs_from_model(self.fake, torch.bfloat16), r, r)

    def critic_state(self):
        return {"heads": self.heads.state_dict(), "head_optimizer": self.opt_h.state_dict(),
                "gap_ema": self.gap.gap_ema.cpu(), "gap_cnt": self.gap.gap_ready.cpu(),
                "ema_banks": [b.state_dict() for b in self.ema_banks], "student_steps": self.student_steps}

    def load_critic_state(self, sd):
        self.heads.load_state_dict(sd["heads"])
        self.opt_h.load_state_dict(sd["head_optimizer"])
        self.gap.gap_ema.copy_(sd["gap_ema"])
        self.gap.gap_ready.copy_(sd["gap_cnt"])
        for b, s in zip(self.ema_banks, sd["ema_banks"]):
            b.load_state_dict(s)
        self.student_steps = sd["student_steps"]
