"""Reference arm of bench.py: the reference's own Wan DMAD workload on the reference's own code.

What runs (all imported, unmodified, from the installed copy in baseline/_ref):
  * the networks: ``rcm.networks.wan2pt1.WanModel`` with the 1.3B shape and the reference's
    block-wise activation checkpointing (``SACConfig(mode="block_wise")``, as its 1.3B rCM/DMAD
    experiment configures both the student and the critic), i.e. its cuDNN-SDPA attention,
    fp32-autocast norms and RoPE;
  * the time utilities ``rcm.utils.timestep_utils`` (UniformShift p_D, RF/TrigFlow conversions)
    and the preconditioning ``rcm.utils.denoiser_scaling.RectifiedFlow_TrigFlowWrapper``;
  * the EMA updater ``imaginaire.utils.ema.FastEmaModelUpdater``.
The DMAD model class itself (rcm/models/t2v_model_distill_dmad.py) cannot be imported here: its
module chain needs omegaconf, hydra and megatron-core, which are not installed.  This file
therefore performs the same sequence of calls as that class's ``_student_dmad_step``,
``training_step_critic`` and ``backward_simulation`` (and the trainer's optimiser / EMA hooks),
with the critic heads, frozen-gain spectral norm and master-weight AdamW written with plain
torch APIs exactly as the reference registers them.  None of dmad_b200's models, kernels or
engine is used on this path.

Install (the reference ships no packaging metadata; ``provision`` does this when baseline/_ref is missing and
the reference checkout is on the machine): copy train/wan/{rcm,imaginaire} to a scratch directory, add a
pyproject.toml, then
    python -m pip install --no-index --no-build-isolation --no-deps --target baseline/_ref <copy>
"""
from __future__ import annotations

import json
import math
import os
import sys

import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
NUM_GAP_BANDS = 10


def _unavailable(msg):
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": msg}))


def _sn_wrap_linear(mod, power_iters=30, allow_frozen=False):
    """Frozen-gain spectral norm registered as the reference does (t2v_model_distill_dmad.py:488-507)."""
    from torch.nn.utils import parametrize
    from torch.nn.utils.parametrizations import spectral_norm

    w = getattr(mod, "weight", None)
    if not isinstance(w, nn.Parameter) or w.dim() != 2 or (not w.requires_grad and not allow_frozen):
        return 0
    if torch.linalg.matrix_norm(w.detach().float(), ord=2) < 1e-8:
        return 0
    w_orig = w.detach().clone()
    spectral_norm(mod, name="weight", n_power_iterations=1)
    with torch.no_grad():
        for _ in range(power_iters):
            _ = mod.weight
        wn = mod.weight.detach()
        gain = (w_orig.flatten().float() @ wn.flatten().float()) / (wn.flatten().float() @ wn.flatten().float())

    class _FrozenGain(nn.Module):
        def __init__(self, g):
            super().__init__()
            self.register_buffer("gain", g)

        def forward(self, x):
            return x * self.gain

    parametrize.register_parametrization(mod, "weight", _FrozenGain(gain.to(w_orig.dtype)))
    return 1


def _stub_log_colours():
    """``termcolor`` (log colours only) is not in this image; the reference's ``imaginaire.utils.misc``
    imports it at module level.  A stand-in that returns the text uncoloured lets the reference's own
    optimiser module import unmodified."""
    import types

    try:
        import termcolor  # noqa: F401
    except ImportError:
        mod = types.ModuleType("termcolor")
        mod.colored = lambda text, *a, **k: text
        sys.modules["termcolor"] = mod


class ReferenceWanDMAD:
    def __init__(self, device, layers=None, seed=0):
        sys.path.insert(0, REF)
        _stub_log_colours()
        from imaginaire.utils.ema import FastEmaModelUpdater
        from rcm.utils.fused_adam_dtensor import MasterWeightAdamW
        from rcm.networks.wan2pt1 import WanModel
        from rcm.utils.denoiser_scaling import RectifiedFlow_TrigFlowWrapper
        from rcm.utils.selective_activation_checkpoint import SACConfig
        from rcm.utils.timestep_utils import UniformShift, rf_to_trig_time, trig_to_rf_time

        self.rf_to_trig_time, self.trig_to_rf_time = rf_to_trig_time, trig_to_rf_time
        net_args = dict(dim=1536, eps=1e-06, ffn_dim=8960, freq_dim=256, in_dim=16, num_heads=12,
                        num_layers=layers or 30, out_dim=16, text_len=512, model_type="t2v")
        torch.manual_seed(seed)
        with torch.device(device):
            self.net = WanModel(**net_args, sac_config=SACConfig(mode="block_wise"))
            self.net_fake_score = WanModel(**net_args, sac_config=SACConfig(mode="block_wise"))
            self.net_fake_score.load_state_dict(self.net.state_dict())
            self.net_ema = WanModel(**net_args, sac_config=SACConfig(mode="block_wise"))
            dim = 1536

            def _head():
                return nn.Sequential(nn.Linear(dim, dim), nn.SiLU(), nn.Linear(dim, 1))

            self.heads = nn.ModuleDict({"real": _head(), "teacher": _head()}).float()
        if torch.device(device).type == "cuda":
            for net in (self.net, self.net_fake_score, self.net_ema):
                net.disable_context_parallel()
        # spectral norm: every critic block Linear and head; first half of the generator and its EMA
        for module in (self.net_fake_score.blocks, self.heads):
            for m in module.modules():
                if isinstance(m, nn.Linear):
                    _sn_wrap_linear(m)
        self.net_ema.requires_grad_(False)
        for net in (self.net, self.net_ema):
            nb = math.ceil(len(net.blocks) * 0.5)
            for block in list(net.blocks)[:nb]:
                for m in block.modules():
                    if isinstance(m, nn.Linear):
                        _sn_wrap_linear(m, allow_frozen=True)
        self.ema = FastEmaModelUpdater()
        self.ema.copy_to(src_model=self.net, tgt_model=self.net_ema)
        # on_train_start: nets in bf16, EMA in fp32
        self.net.to(dtype=torch.bfloat16)
        self.net_fake_score.to(dtype=torch.bfloat16)
        self.net_ema.to(dtype=torch.float32)
        self.net.train()
        self.net_fake_score.train()
        s = 0.1
        import numpy as np

        self.ema_coef = float(np.roots([1, 7, 16 - s ** -2, 12 - s ** -2]).real.max())
        self.scaling = RectifiedFlow_TrigFlowWrapper(1.0, 1000.0)
        self.p_D = UniformShift(shift=5.0)
        self.device = device
        self._gap_ema = torch.zeros(NUM_GAP_BANDS, device=device)
        self._gap_ready = torch.zeros(NUM_GAP_BANDS, device=device)
        kw = dict(lr=2e-6, betas=(0.0, 0.99), eps=1e-8, weight_decay=0.01)
        # the reference's own master-weight AdamW (fused_adam_dtensor.py:372-416), which its optimiser
        # factory selects when Transformer Engine is absent (as here)
        self.opt_net = MasterWeightAdamW([p for p in self.net.parameters() if p.requires_grad], **kw)
        self.opt_fake = MasterWeightAdamW([p for p in self.net_fake_score.parameters() if p.requires_grad]
                                          + list(self.heads.parameters()), **kw)
        self.params_net = [p for g in self.opt_net.param_groups for p in g["params"]]
        self.params_fake = [p for g in self.opt_fake.param_groups for p in g["params"]]
        self.world = torch.distributed.get_world_size() if torch.distributed.is_initialized() else 1

    # ------------------------------------------------------------------ rcm model pieces
    def draw_time_D(self, n):
        return self.rf_to_trig_time(self.p_D(shape=(n, 1), device=self.device, dtype=torch.float64).clamp(0.0, 1.0))

    def denoise(self, net, xt, time, ctx):
        time_B_T = time.reshape(-1, 1)
        t5 = time_B_T.reshape(-1, 1, 1, 1, 1)
        c_skip, c_out, c_in, c_noise = self.scaling(trigflow_t=t5)
        out = net(x_B_C_T_H_W=(xt * c_in).to(device=self.device, dtype=torch.bfloat16),
                  timesteps_B_T=c_noise.squeeze(dim=[1, 3, 4]).to(device=self.device, dtype=torch.bfloat16),
                  crossattn_emb=ctx).float()
        return c_skip * xt + c_out * out

    def backward_simulation(self, ctx, size, n_steps, with_grad):
        G_time = math.pi / 2 * torch.ones(size[0], 1, device=self.device)
        x = torch.randn(size, device=self.device)
        t_traj = [G_time]
        for _ in range(n_steps - 1):
            G_time = torch.minimum(self.draw_time_D(size[0]), G_time)
            t_traj.append(G_time)
        t_traj.append(0 * G_time)
        for step, (tc, tn) in enumerate(zip(t_traj[:-1], t_traj[1:])):
            fn = torch.enable_grad if with_grad and step == n_steps - 1 else torch.no_grad
            with fn():
                x = self.denoise(self.net, x, tc, ctx).float()
            if step < n_steps - 1:
                tn5 = tn.reshape(-1, 1, 1, 1, 1)
                x = torch.cos(tn5) * x + torch.sin(tn5) * torch.randn_like(x)
        return x

    def critic_forward(self, xt, t, ctx):
        feats = []
        h = self.net_fake_score.blocks[-1].register_forward_hook(lambda m, i, o: feats.append(o))
        try:
            x0 = self.denoise(self.net_fake_score, xt, t, ctx)
        finally:
            h.remove()
        tok = feats[-1].float()
        d_r = self.heads["real"](tok).mean(dim=1).squeeze(-1)
        d_t = self.heads["teacher"](tok).mean(dim=1).squeeze(-1)
        return x0, d_r, d_t

    def noise_D(self, x0, t):
        eps = torch.randn(x0.size(), device=self.device)
        tt = t.reshape(-1, 1, 1, 1, 1)
        return torch.cos(tt) * x0 + torch.sin(tt) * eps

    def gap_band(self, t):
        u = self.p_D.cdf_rf(self.trig_to_rf_time(t.reshape(-1).to(torch.float64)))
        return (u * NUM_GAP_BANDS).long().clamp(0, NUM_GAP_BANDS - 1)

    def gap_weight(self, t):
        ready = self._gap_ready > 0
        if int(ready.sum()) < 5:
            return None, 1.0
        center = float(self._gap_ema[ready].median())
        w_band = torch.sigmoid((center - self._gap_ema) / 2.0)
        return w_band[self.gap_band(t)], float(w_band[ready].mean().clamp(min=1e-3))

    @torch.no_grad()
    def update_gap(self, dT, dQ, tT, tQ):
        bt, bq = self.gap_band(tT), self.gap_band(tQ)
        sT = torch.zeros(NUM_GAP_BANDS, device=self.device).scatter_add_(0, bt, dT.float())
        cT = torch.zeros(NUM_GAP_BANDS, device=self.device).scatter_add_(0, bt, torch.ones_like(dT))
        sQ = torch.zeros(NUM_GAP_BANDS, device=self.device).scatter_add_(0, bq, dQ.float())
        cQ = torch.zeros(NUM_GAP_BANDS, device=self.device).scatter_add_(0, bq, torch.ones_like(dQ))
        if self.world > 1:
            for t in (sT, cT, sQ, cQ):
                torch.distributed.all_reduce(t)
        valid = (cT > 0) & (cQ > 0)
        now = sT / cT.clamp(min=1) - sQ / cQ.clamp(min=1)
        upd = torch.where(valid & (self._gap_ready > 0), 0.99 * self._gap_ema + 0.01 * now, now)
        self._gap_ema.copy_(torch.where(valid, upd, self._gap_ema))
        self._gap_ready.copy_(torch.where(valid, torch.ones_like(self._gap_ready), self._gap_ready))

    def _sync_grads(self, params):
        if self.world > 1:
            for p in params:
                if p.grad is not None:
                    torch.distributed.all_reduce(p.grad)
                    p.grad.div_(self.world)

    # ------------------------------------------------------------------ trainer iteration
    def training_step(self, batch, it):
        ctx = batch["context"]
        x0 = batch["latents"]
        if it % 2 == 0:  # student phase
            eff = it // 2
            n_sim = eff % 4 + 1
            G = self.backward_simulation(ctx, x0.size(), n_sim, True)
            D = self.draw_time_D(x0.shape[0])
            xt = self.noise_D(G, D)
            self.net_fake_score.requires_grad_(False)
            self.heads.requires_grad_(False)
            _, d_r, d_t = self.critic_forward(xt, D, ctx)
            w, E_w = self.gap_weight(D)
            tterm = -d_t if w is None else -d_t * w / E_w
            loss = tterm - d_r
            loss.sum().backward()
            self.net_fake_score.requires_grad_(True)
            self.heads.requires_grad_(True)
            self._sync_grads(self.params_net)
            torch.nn.utils.clip_grad_norm_(self.params_net, 1e12, foreach=True)
            self.opt_net.step()
            beta = 0.0 if eff < 1 else (1 - 1 / (eff + 1)) ** (self.ema_coef + 1)
            self.ema.update_average(self.net, self.net_ema, beta=beta)
            self.opt_net.zero_grad(set_to_none=True)
            return {"dmad_g_loss": loss.detach().mean()}
        eff_fake = it - it // 2 - 1
        n_sim = eff_fake % 4 + 1
        G = self.backward_simulation(ctx, x0.size(), n_sim, False)
        D = self.draw_time_D(x0.shape[0])
        xt_G = self.noise_D(G, D)
        _, d_r_G, d_t_G = self.critic_forward(xt_G, D, ctx)
        _, d_r_Q, d_t_Q = self.critic_forward(self.noise_D(x0, D), D, ctx)
        _, d_r_T, _ = self.critic_forward(self.noise_D(batch["real_latents"], D), D, ctx)
        bce = F.softplus(-d_t_Q) + F.softplus(d_t_G) + F.softplus(-d_r_T) + F.softplus(d_r_G)
        bce.sum().backward()
        self.update_gap(d_r_T.detach(), d_r_Q.detach(), D, D)
        self._sync_grads(self.params_fake)
        torch.nn.utils.clip_grad_norm_(self.params_fake, 1e12, foreach=True)
        self.opt_fake.step()
        self.opt_fake.zero_grad(set_to_none=True)
        return {"dmad_d_loss": bce.detach().mean()}

    @torch.no_grad()
    def generate(self, ctx, shape, num_steps=4):
        mid_t = [1.5, 1.4, 1.0][: num_steps - 1]
        t_steps = torch.tensor([math.atan(80.0)] + mid_t + [0.0], dtype=torch.float64, device=self.device)
        x = torch.randn(shape, device=self.device, dtype=torch.float32).to(torch.float64)
        ones = torch.ones(shape[0], device=self.device, dtype=torch.float64)
        self.net.eval()
        for tc, tn in zip(t_steps[:-1], t_steps[1:]):
            x = self.denoise(self.net, x.float(), tc.float() * ones, ctx).to(torch.float64)
            x = torch.cos(tn) * x + torch.sin(tn) * torch.randn(shape, device=self.device)
        self.net.train()
        return torch.nan_to_num(x.float())


_PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "dmad-reference-wan"
version = "0.0.0"

[tool.setuptools.packages.find]
include = ["rcm*", "imaginaire*"]
"""


def _reference_checkout():
    try:
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            path = json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None
    return path if path and os.path.isdir(os.path.join(path, "train", "wan", "rcm")) else None


def provision(log=sys.stderr) -> bool:
    """Installs the unmodified reference into baseline/_ref when it is missing and the reference checkout
    (BASELINE.json's ``reference_path``) is on this machine: ``train/wan/{rcm,imaginaire}`` copied to a
    scratch directory with packaging metadata added, ``pip install --no-index --no-deps --target``, and
    ``train/image/{main,third_party}`` copied beside them.  Returns whether baseline/_ref is in place."""
    if os.path.isdir(os.path.join(REF, "rcm", "networks")):
        return True
    src = _reference_checkout()
    if src is None:
        return False
    import shutil
    import subprocess
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        for name in ("rcm", "imaginaire"):
            shutil.copytree(os.path.join(src, "train", "wan", name), os.path.join(tmp, name))
        with open(os.path.join(tmp, "pyproject.toml"), "w") as f:
            f.write(_PYPROJECT)
        print(f"# installing the reference from {src} into {REF}", file=log, flush=True)
        rc = subprocess.call([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                              "--target", REF, tmp], stdout=log, stderr=log)
    if rc != 0:
        return False
    for name in ("main", "third_party"):
        dst = os.path.join(REF, "image", name)
        if not os.path.isdir(dst):
            shutil.copytree(os.path.join(src, "train", "image", name), dst)
    return os.path.isdir(os.path.join(REF, "rcm", "networks"))


def build_reference_trainer(args, device):
    if not provision():
        _unavailable("baseline/_ref missing and no reference checkout to install it from: the reference has no "
                     "setup.py/pyproject.toml, so it is installed from a copy with packaging metadata added")
        return None
    return ReferenceWanDMAD(device, layers=args.layers)
