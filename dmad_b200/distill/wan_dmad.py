"""DMAD distillation of a Wan2.1-shaped DiT (rCM's distillation model with the DMD term
replaced by the two-head critic; no sCM loss).

Parity with train/wan/rcm/models/t2v_model_distill_dmad.py and the rCM base class
(train/wan/rcm/models/t2v_model_distill_rcm.py):
* nets: student ``net`` (few-step generator), critic backbone ``net_fake_score`` (a copy of the
  teacher) with ``CriticHeads`` on the token output of its last block, fp32 power-EMA of the student;
* G / Q / T share one TrigFlow time drawn from p_D per sample, with independent noise
  (``_noise_with_D_time``, dmad :344-352);
* student step: backward simulation with 1..4 student evaluations (only the last carries grad,
  rcm :514-542), critic frozen, loss ``-d_real(G) - w_gap d_teacher(G)`` (dmad :399-426);
* critic step: no-grad backward simulation, three critic forwards, softplus BCE, all-reduced gap
  EMA over CDF-decile bands of p_D (dmad :437-469, :356-395);
* generator and critic alternate 1:1 (``student_update_freq=2``, rcm :297-311);
* frozen-gain spectral norm on every critic block Linear and head, and on the first half of the
  generator's blocks (dmad :488-517);
* few-step sampler ``x <- cos(t') x0 + sin(t') eps`` from t = atan(sigma_max) (rcm :830-895).

The critic's three forwards are run forward+backward one at a time (the gradient of the summed
BCE is identical), so activations of only one forward are alive at once.
"""
from __future__ import annotations

import contextlib
import copy
import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn

from ..algorithms import (CriticHeads, GapRouter, TrigFlowScaling, UniformShift, LogNormal, critic_bce_loss,
                          ema_exp_coefficient, generator_linear_loss, rf_to_trig_time, trig_to_rf_time)
from ..algorithms.dmad import band_of_cdf, critic_accuracies
from ..algorithms.spectral import apply_spectral_norm
from ..models.wan import WanConfig, WanModel, WAN_1P3B
from ..ops.optim import FusedAdamW
from ..parallel.dist import broadcast_module
from ..parallel.dp import GradSync
from ..parallel.zero import ShardedAdamW


@dataclass
class WanDMADConfig:
    net: WanConfig = field(default_factory=lambda: WanConfig(**WAN_1P3B.__dict__))
    sigma_max: float = 80.0
    p_D_shift: float = 5.0          # p_D = UniformShift(5) (rcm 1.3B experiment)
    p_D_lognormal: tuple | None = None  # (mean, std) to use LogNormal instead
    max_simulation_steps_fake: int = 4
    student_update_freq: int = 2
    backward_timesteps: tuple = (1.5, 1.4, 1.0)
    dmd_fix_timesteps: bool = False
    loss_scale_dmd: float = 1.0
    critic_spectral_norm: bool = True
    generator_spectral_norm: bool = True
    sn_generator_frac: float = 0.5
    sn_power_iters: int = 30
    gap_route: bool = True
    gap_tau: float = 2.0
    gap_ema_beta: float = 0.99
    lr: float = 2e-6
    critic_lr: float = 2e-6
    betas: tuple = (0.0, 0.99)
    weight_decay: float = 0.01
    eps: float = 1e-8
    ema_enabled: bool = True
    ema_rate: float = 0.1
    grad_clip: float | None = None  # rcm grad_clip=False: no clipping (max norm 1e12)
    grad_force_finite: bool = True  # the default GradClip(force_finite=True) callback: nan/inf grads -> 0
    student_lora_rank: int = 0
    checkpoint_student_blocks: int = 0
    checkpoint_critic_blocks: int = 0
    checkpoint_critic_blocks_student_phase: int | None = None
    checkpoint_student_policy: str = "block_wise"  # "mm_only": keep matmul / attention outputs
    checkpoint_critic_policy: str = "block_wise"
    rectified_flow_t_scaling_factor: float = 1000.0
    # rCM consistency term (0 = pure DMAD, as the reference's DMAD experiments; > 0 adds the sCM /
    # dCM loss of the rCM recipe in the student phase, which needs the teacher network)
    loss_scale: float = 0.0
    cm_type: str = "scm"            # "scm" | "dcm"
    use_rf_scm: bool = False
    teacher_guidance: float = 5.0
    tangent_warmup: int = 0
    p_G_lognormal: tuple = (0.7, 1.6)
    fd_type: int = 0
    fd_size: float = 1e-4
    dcm_total_steps: int = 48
    dcm_skipping_interval_steps: int = 1
    dcm_timestep_shift: float = 5.0
    # "dmad": two-head GAN critic (this model); "dmd": rCM's DMD with a denoising fake score
    critic_mode: str = "dmad"
    # "sharded": flat symmetric buffers + one fused reduce-scatter / AdamW / all-gather kernel per
    # step (fp32 optimiser state sharded over the ranks); "replicated": NCCL all-reduce of the
    # gradients, then the same multi-tensor AdamW on every rank
    # shard the frozen block weights (LoRA student base, teacher) over the ranks and gather them one
    # block ahead (needs the student blocks activation-checkpointed)
    shard_frozen: bool = False
    # FSDP-style sharding of the trainable block weights (critic, and the student unless it is a LoRA
    # student): bf16 shards gathered one block ahead, gradients reduce-scattered per block in backward,
    # AdamW on the shards; the blocks are then activation-checkpointed
    fsdp_trainable: bool = False
    # hybrid sharding (HSDP): shard the block weights over groups of this many consecutive ranks and
    # replicate across the groups (None: shard over all ranks)
    fsdp_shard_size: int | None = None
    dp_optimizer: str = "sharded"
    dp_multicast: bool = True
    dp_sync_timeout_s: float = 120.0
    # pretrained teacher: a DCP directory, a release / plain .pth or a .safetensors file; student and
    # critic backbone start from it (rcm :197-251); None = random init
    teacher_ckpt: str | None = None


class WanDMAD(nn.Module):
    def __init__(self, cfg: WanDMADConfig, device=None, dtype=torch.bfloat16, seed: int = 0):
        super().__init__()
        self.cfg = cfg
        self.dtype = dtype
        device = torch.device(device) if device is not None else torch.device("cpu")
        torch.manual_seed(seed)
        if device.type == "cuda":
            # built on the device in the compute dtype: a 14B net is 28 GB there, and three fp32 host copies
            # per rank would not fit in host memory
            with torch.device(device):
                teacher = WanModel(cfg.net)
            teacher.to(dtype)
        else:
            teacher = WanModel(cfg.net)
        if cfg.teacher_ckpt:
            from ..tools.import_reference_checkpoint import read_pretrained
            res = teacher.load_state_dict(read_pretrained(cfg.teacher_ckpt), strict=False)
            if res.missing_keys:
                raise KeyError(f"teacher checkpoint {cfg.teacher_ckpt} lacks {len(res.missing_keys)} weights, "
                               f"e.g. {res.missing_keys[:3]}")
        # student and critic backbone both start from the teacher weights (rcm :247-251)
        self.net = teacher
        self.net_fake_score = copy.deepcopy(teacher)
        need_teacher = cfg.loss_scale > 0 or cfg.critic_mode == "dmd"
        self.net_teacher = copy.deepcopy(teacher).requires_grad_(False) if need_teacher else None
        self.critic_heads = CriticHeads(cfg.net.dim)
        if cfg.critic_spectral_norm:
            self.net_fake_score.enable_spectral_norm(range(cfg.net.num_layers), cfg.sn_power_iters)
            apply_spectral_norm(self.critic_heads, cfg.sn_power_iters, types=(nn.Linear,))
        if cfg.generator_spectral_norm:
            nb = math.ceil(cfg.net.num_layers * cfg.sn_generator_frac)
            self.net.enable_spectral_norm(range(nb), cfg.sn_power_iters)
        if cfg.student_lora_rank:
            self.net.enable_lora(cfg.student_lora_rank)
        self.net.to(device=device, dtype=dtype)
        self.net_fake_score.to(device=device, dtype=dtype)
        if self.net_teacher is not None:
            self.net_teacher.to(device=device, dtype=dtype).eval()
            broadcast_module(self.net_teacher)
        self.critic_heads.to(device=device, dtype=torch.float32)
        self.net.checkpoint_blocks = cfg.checkpoint_student_blocks
        self.net_fake_score.checkpoint_blocks = cfg.checkpoint_critic_blocks
        self.net.checkpoint_policy = cfg.checkpoint_student_policy
        self.net_fake_score.checkpoint_policy = cfg.checkpoint_critic_policy
        broadcast_module(self.net)
        broadcast_module(self.net_fake_score)
        broadcast_module(self.critic_heads)
        self.sharded = []
        if cfg.shard_frozen:
            from ..parallel.fsdp import ShardedFrozenBlocks
            if cfg.student_lora_rank:
                sh = ShardedFrozenBlocks(self.net.blocks)
                sh.check_checkpointing(cfg.checkpoint_student_blocks)
                self.sharded.append(sh)
            if self.net_teacher is not None:
                self.sharded.append(ShardedFrozenBlocks(self.net_teacher.blocks))
        self.fsdp = {}
        if cfg.fsdp_trainable:
            from ..parallel.dist import get_world_size
            from ..parallel.fsdp import ShardedTrainableBlocks, hsdp_groups
            if cfg.dp_optimizer != "sharded":
                raise ValueError("fsdp_trainable runs with dp_optimizer='sharded'")
            shard_group = rep_group = None
            if cfg.fsdp_shard_size and cfg.fsdp_shard_size < get_world_size():
                shard_group, rep_group = hsdp_groups(cfg.fsdp_shard_size)
            kw_b = dict(betas=cfg.betas, eps=cfg.eps, weight_decay=cfg.weight_decay,
                        sync_timeout_s=cfg.dp_sync_timeout_s, force_finite=cfg.grad_force_finite,
                        group=shard_group, replicate_group=rep_group)
            nl = cfg.net.num_layers
            cfg.checkpoint_critic_blocks = cfg.checkpoint_critic_blocks_student_phase = nl
            self.net_fake_score.checkpoint_blocks = nl
            self.fsdp["critic"] = ShardedTrainableBlocks(self.net_fake_score.blocks, lr=cfg.critic_lr, **kw_b)
            if not cfg.student_lora_rank:
                cfg.checkpoint_student_blocks = nl
                self.net.checkpoint_blocks = nl
                self.fsdp["student"] = ShardedTrainableBlocks(self.net.blocks, lr=cfg.lr, ema=cfg.ema_enabled, **kw_b)
        self.gap = GapRouter("allreduce", tau=cfg.gap_tau, beta=cfg.gap_ema_beta, enabled=cfg.gap_route).to(device)
        self.scaling = TrigFlowScaling(1.0, cfg.rectified_flow_t_scaling_factor)
        self.p_D = LogNormal(*cfg.p_D_lognormal) if cfg.p_D_lognormal else UniformShift(cfg.p_D_shift)
        self.device = device
        # optimisers; the student's optimiser also advances the fp32 EMA copy in the same kernel pass
        s_params = [p for p in self.net.parameters() if p.requires_grad]
        self._student_params = s_params  # the EMA's order
        c_params = [p for p in self.net_fake_score.parameters() if p.requires_grad] + list(self.critic_heads.parameters())
        self.ema_coef = ema_exp_coefficient(cfg.ema_rate)
        if cfg.dp_optimizer == "sharded":
            kw = dict(betas=cfg.betas, eps=cfg.eps, weight_decay=cfg.weight_decay, use_multicast=cfg.dp_multicast,
                      sync_timeout_s=cfg.dp_sync_timeout_s, force_finite=cfg.grad_force_finite)

            def make(params, lr, ema, name):
                sh = self.fsdp.get(name)
                if sh is None:
                    return ShardedAdamW(params, lr=lr, ema=ema, **kw)
                from ..parallel.fsdp import FSDPOptimizer
                owned = {id(p) for p in sh.params}
                rest = [p for p in params if id(p) not in owned]
                return FSDPOptimizer(sh, ShardedAdamW(rest, lr=lr, ema=ema, **kw) if rest else None)

            self.opt_student = make(s_params, cfg.lr, cfg.ema_enabled, "student")
            self.opt_critic = make(c_params, cfg.critic_lr, False, "critic")
            self.ema_params = None
            self.sync_student = GradSync(s_params, enabled=False)
            self.sync_critic = GradSync(c_params, enabled=False)
        elif cfg.dp_optimizer == "replicated":
            self.ema_params = [p.detach().float().clone() for p in s_params] if cfg.ema_enabled else None
            self.opt_student = FusedAdamW(s_params, lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                          weight_decay=cfg.weight_decay, ema=self.ema_params)
            self.opt_critic = FusedAdamW(c_params, lr=cfg.critic_lr, betas=cfg.betas, eps=cfg.eps,
                                         weight_decay=cfg.weight_decay)
            self.sync_student = GradSync(s_params)
            self.sync_critic = GradSync(c_params)
        else:
            raise ValueError(f"unknown dp_optimizer {cfg.dp_optimizer!r}")

    # ------------------------------------------------------------------ trainer interface
    def phase_of(self, it: int) -> str:
        return "student" if self.is_student_phase(it) else "critic"

    def optimizers(self) -> dict:
        return {"student": self.opt_student, "critic": self.opt_critic}

    def context_parallel_nets(self) -> list:
        return [n for n in (self.net, self.net_fake_score, self.net_teacher) if n is not None]

    # ------------------------------------------------------------------ checkpoint state
    def _full_blocks(self, write_back=False):
        """Context with every FSDP-sharded block weight gathered into full tensors (collective)."""
        stack = contextlib.ExitStack()
        for sh in self.fsdp.values():
            stack.enter_context(sh.materialized(write_back))
        return stack

    def state_dicts(self) -> tuple[dict, dict | None]:
        """(state every rank holds identically, this rank's optimiser shards or None)."""
        with self._full_blocks():
            # sharded frozen weights are never saved (they do not change; they come from the teacher checkpoint)
            net_sd = {k: v.clone() for k, v in self.net.state_dict().items() if v.numel() > 0 or not self.sharded}
            shared = {"net": net_sd, "net_fake_score": {k: v.clone() for k, v in self.net_fake_score.state_dict().items()},
                      "critic_heads": self.critic_heads.state_dict(), "gap": self.gap.state_dict()}
        if self.fsdp:
            return shared, {"opt_student": self.opt_student.state_dict(), "opt_critic": self.opt_critic.state_dict()}
        if isinstance(self.opt_student, ShardedAdamW):
            names = {id(p): n for n, p in self.net.named_parameters()}
            shared["student_layout"] = self.opt_student.layout(names)
            return shared, {"opt_student": self.opt_student.state_dict(), "opt_critic": self.opt_critic.state_dict()}
        shared["opt_student"] = self.opt_student.state_dict()
        shared["opt_critic"] = self.opt_critic.state_dict()
        shared["ema"] = self.ema_params
        return shared, None

    def load_state_dicts(self, shared: dict, per_rank: dict | None):
        with self._full_blocks(write_back=True):
            self.net.load_state_dict(shared["net"], strict=not self.sharded)
            self.net_fake_score.load_state_dict(shared["net_fake_score"])
        self.critic_heads.load_state_dict(shared["critic_heads"])
        self.gap.load_state_dict(shared["gap"])
        if self.fsdp:
            if not per_rank or "opt_student" not in per_rank or "elastic_rank_states" in per_rank:
                raise RuntimeError("an FSDP-sharded run resumes from its own per-rank shards at the same world size")
            self.opt_student.load_state_dict(per_rank["opt_student"])
            self.opt_critic.load_state_dict(per_rank["opt_critic"])
            return
        if isinstance(self.opt_student, ShardedAdamW):
            if per_rank and "elastic_rank_states" in per_rank:  # saved with another world size
                states = per_rank["elastic_rank_states"]
                self.opt_student.load_resharded([st["opt_student"] for st in states])
                self.opt_critic.load_resharded([st["opt_critic"] for st in states])
                return
            if not per_rank or "opt_student" not in per_rank:
                raise RuntimeError("checkpoint has no per-rank optimiser shards (saved with a replicated optimiser)")
            self.opt_student.load_state_dict(per_rank["opt_student"])
            self.opt_critic.load_state_dict(per_rank["opt_critic"])
        else:
            self.opt_student.load_state_dict(shared["opt_student"])
            self.opt_critic.load_state_dict(shared["opt_critic"])
            if self.ema_params is not None and shared.get("ema") is not None:
                for d, s_ in zip(self.ema_params, shared["ema"]):
                    d.copy_(s_)

    def ema_weights(self) -> list[torch.Tensor] | None:
        """Full fp32 EMA of the student's trainable parameters (collective when sharded)."""
        if "student" in self.fsdp:
            by = self.opt_student.full_ema_by_param()
            return None if by is None else [by[id(p)] for p in self._student_params]
        if isinstance(self.opt_student, ShardedAdamW):
            return self.opt_student.full_ema()
        return self.ema_params

    # ------------------------------------------------------------------ schedule (rcm :297-311)
    def is_student_phase(self, it: int) -> bool:
        w = self.cfg.tangent_warmup
        return it < w or (it - w) % self.cfg.student_update_freq == 0

    def effective_iteration(self, it: int) -> int:
        w = self.cfg.tangent_warmup
        return it if it < w else w + (it - w) // self.cfg.student_update_freq

    def effective_iteration_fake(self, it: int) -> int:
        return it - self.effective_iteration(it) - 1

    def ema_beta(self, it: int) -> float:
        if it < 1:
            return 0.0
        return (1 - 1 / (it + 1)) ** (self.ema_coef + 1)

    # ------------------------------------------------------------------ time draws
    def draw_time_D(self, n: int):
        rf = self.p_D((n, 1), device=self.device, dtype=torch.float64).clamp(0.0, 1.0)
        return rf_to_trig_time(rf)

    def gap_band(self, t_trig):
        return band_of_cdf(self.p_D.cdf_rf(trig_to_rf_time(t_trig.reshape(-1).to(torch.float64))))

    # ------------------------------------------------------------------ denoiser
    def _net_timesteps(self, c_noise):
        # the reference hands the network bf16 timesteps (rcm :438-441)
        return c_noise.to(self.dtype).float()

    def denoise(self, net, xt, t_B_1, context):
        """x0 prediction of ``net`` at TrigFlow time t (uniform per sample)."""
        t5 = t_B_1.reshape(-1, 1, 1, 1, 1).to(torch.float64)
        c_skip, c_out, c_in, c_noise = self.scaling(t5)
        out = net((xt * c_in).to(self.dtype), self._net_timesteps(c_noise.reshape(-1, 1)), context).float()
        return (c_skip * xt + c_out * out).float()

    def critic_forward(self, xt, t_B_1, context, need_x0=False):
        """(x0 or None, d_real [B], d_teacher [B]) from the critic backbone's last-block tokens."""
        net = self.net_fake_score
        t5 = t_B_1.reshape(-1, 1, 1, 1, 1).to(torch.float64)
        c_skip, c_out, c_in, c_noise = self.scaling(t5)
        xin = (xt * c_in).to(self.dtype)
        ts = self._net_timesteps(c_noise.reshape(-1, 1))
        if need_x0:
            out, feats = net(xin, ts, context, feature_hook_block=-1)
            x0 = (c_skip * xt + c_out * out.float()).float()
        else:
            feats = net(xin, ts, context, stop_after_block=len(net.blocks) - 1)
            x0 = None
        d_real, d_teacher = self.critic_heads.pooled(feats)
        cp = net.cp
        if cp is not None and cp.world > 1:
            # mean over this rank's tokens, summed over the CP group / cp (dmad :338-339)
            d_real = cp.all_reduce_sum(d_real) / cp.world
            d_teacher = cp.all_reduce_sum(d_teacher) / cp.world
        return x0, d_real, d_teacher

    # ------------------------------------------------------------------ backward simulation (rcm :514-542)
    def backward_simulation(self, context, shape, n_steps: int, with_grad: bool):
        B = shape[0]
        t = torch.full((B, 1), math.pi / 2, device=self.device, dtype=torch.float64)
        x = torch.randn(shape, device=self.device)
        traj = [t]
        for i in range(n_steps - 1):
            if self.cfg.dmd_fix_timesteps:
                t = torch.full((B, 1), self.cfg.backward_timesteps[i], device=self.device, dtype=torch.float64)
            else:
                t = torch.minimum(self.draw_time_D(B), t)
            traj.append(t)
        traj.append(torch.zeros_like(t))
        for step, (tc, tn) in enumerate(zip(traj[:-1], traj[1:])):
            grad_on = with_grad and step == n_steps - 1
            with torch.set_grad_enabled(grad_on):
                x = self.denoise(self.net, x, tc, context)
            if step < n_steps - 1:
                tn5 = tn.reshape(-1, 1, 1, 1, 1)
                x = torch.cos(tn5) * x + torch.sin(tn5) * torch.randn_like(x)
                x = x.float()
        return x

    def _noise(self, x0, t_B_1):
        eps = torch.randn(x0.shape, device=self.device)
        t5 = t_B_1.reshape(-1, 1, 1, 1, 1)
        return (torch.cos(t5) * x0 + torch.sin(t5) * eps).float()

    # ------------------------------------------------------------------ steps
    def _set_critic_grad(self, on: bool):
        for p in self.opt_critic.params:
            p.requires_grad_(on)

    def student_step(self, batch, it: int) -> dict:
        cfg = self.cfg
        ctx = batch["context"]
        shape = batch["latents"].shape
        n_sim = self.effective_iteration(it) % cfg.max_simulation_steps_fake + 1
        self.net.train()
        ckpt_stu_phase = cfg.checkpoint_critic_blocks_student_phase
        saved = self.net_fake_score.checkpoint_blocks
        if ckpt_stu_phase is not None:
            self.net_fake_score.checkpoint_blocks = ckpt_stu_phase
        G_x0 = self.backward_simulation(ctx, shape, n_sim, with_grad=True)
        D_time = self.draw_time_D(shape[0])
        xt_G = self._noise(G_x0, D_time)
        self._set_critic_grad(False)
        try:
            _, d_real_G, d_teacher_G = self.critic_forward(xt_G, D_time, ctx)
            w, E_w = self.gap.weights(self.gap_band(D_time))
            loss = cfg.loss_scale_dmd * generator_linear_loss(d_real_G, d_teacher_G, w, E_w)
            loss.sum().backward()
        finally:
            self._set_critic_grad(True)
            self.net_fake_score.checkpoint_blocks = saved
        self.sync_student.sync()
        beta = self.ema_beta(self.effective_iteration(it)) if cfg.ema_enabled else None
        self.opt_student.step(ema_beta=beta, max_grad_norm=cfg.grad_clip)
        self.opt_student.zero_grad()
        out = {"dmad_g_loss": loss.detach().mean(), "dmad_g_d_real": d_real_G.detach().mean(),
               "dmad_g_d_teacher": d_teacher_G.detach().mean(), "n_sim": n_sim}
        if w is not None:
            out["dmad_gap_w_mean"] = w.mean()
            out["dmad_gap_w_norm"] = E_w
        return out

    def critic_step(self, batch, it: int) -> dict:
        cfg = self.cfg
        ctx = batch["context"]
        x0_Q = batch["latents"]
        x0_T = batch["real_latents"]
        shape = x0_Q.shape
        n_sim = self.effective_iteration_fake(it) % cfg.max_simulation_steps_fake + 1
        self.net_fake_score.train()
        with torch.no_grad():
            G_x0 = self.backward_simulation(ctx, shape, n_sim, with_grad=False)
        D_time = self.draw_time_D(shape[0])
        xt_G = self._noise(G_x0, D_time)
        _, d_real_G, d_teacher_G = self.critic_forward(xt_G, D_time, ctx)
        (torch.nn.functional.softplus(d_teacher_G) + torch.nn.functional.softplus(d_real_G)).sum().backward()
        xt_Q = self._noise(x0_Q, D_time)
        _, d_real_Q, d_teacher_Q = self.critic_forward(xt_Q, D_time, ctx)
        torch.nn.functional.softplus(-d_teacher_Q).sum().backward()
        xt_T = self._noise(x0_T, D_time)
        _, d_real_T, _ = self.critic_forward(xt_T, D_time, ctx)
        torch.nn.functional.softplus(-d_real_T).sum().backward()
        bce = critic_bce_loss(d_real_T.detach(), d_real_G.detach(), d_teacher_Q.detach(), d_teacher_G.detach())
        self.gap.update(d_real_T.detach(), d_real_Q.detach(), self.gap_band(D_time), self.gap_band(D_time))
        self.sync_critic.sync()
        self.opt_critic.step(max_grad_norm=cfg.grad_clip)
        self.opt_critic.zero_grad()
        out = {"dmad_d_loss": bce.mean(), "n_sim": n_sim}
        out.update(critic_accuracies(d_real_T, d_real_G, d_teacher_Q, d_teacher_G))
        return out

    def training_step(self, batch, it: int) -> dict:
        from . import rcm

        cfg = self.cfg
        if not self.is_student_phase(it):
            return self.critic_step(batch, it) if cfg.critic_mode == "dmad" else rcm.critic_denoise_step(self, batch, it)
        if cfg.loss_scale > 0:
            return rcm.student_step_with_cm(self, batch, it)
        return self.student_step(batch, it) if cfg.critic_mode == "dmad" else rcm.student_dmd_step(self, batch, it, True)

    # ------------------------------------------------------------------ sampling (rcm :830-895)
    @contextlib.contextmanager
    def ema_scope(self):
        """The student runs with its EMA weights inside (rcm ``ema_scope``); collective when the optimiser
        state is sharded, so every rank enters together."""
        if "student" in self.fsdp:
            sh, rest = self.fsdp["student"], self.opt_student.rest
            if sh.ema is None:
                yield
                return
            rest_ema = rest.full_ema() if rest is not None else None
            saved = [p.detach().clone() for p in rest.params] if rest is not None else []
            with sh.use_weights(sh.ema), torch.no_grad():
                if rest is not None and rest_ema is not None:
                    for p, e in zip(rest.params, rest_ema):
                        p.copy_(e.to(device=p.device, dtype=p.dtype).view_as(p))
                try:
                    yield
                finally:
                    for p, s_ in zip(rest.params if rest is not None else [], saved):
                        p.copy_(s_)
            return
        ema = self.ema_weights()
        if ema is None:
            yield
            return
        params = self._student_params
        saved = [p.detach().clone() for p in params]
        with torch.no_grad():
            for p, e in zip(params, ema):
                p.copy_(e.to(device=p.device, dtype=p.dtype).view_as(p))
        try:
            yield
        finally:
            with torch.no_grad():
                for p, s_ in zip(params, saved):
                    p.copy_(s_)

    @torch.no_grad()
    def generate(self, context, shape, num_steps: int = 4, mid_t=None, generator=None, use_ema=False):
        if use_ema:
            with self.ema_scope():
                return self.generate(context, shape, num_steps, mid_t, generator, use_ema=False)
        cfg = self.cfg
        mid_t = list(mid_t) if mid_t is not None else list(cfg.backward_timesteps[: num_steps - 1])
        t_steps = [math.atan(cfg.sigma_max)] + mid_t + [0.0]
        was = self.net.training
        self.net.eval()
        x = torch.randn(shape, device=self.device, generator=generator, dtype=torch.float32)
        B = shape[0]
        for tc, tn in zip(t_steps[:-1], t_steps[1:]):
            x0 = self.denoise(self.net, x, torch.full((B, 1), tc, device=self.device, dtype=torch.float64), context)
            x = math.cos(tn) * x0 + math.sin(tn) * torch.randn(shape, device=self.device, generator=generator)
        self.net.train(was)
        return torch.nan_to_num(x.float())

