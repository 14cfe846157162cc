"""rCM objectives on the Wan distillation model: sCM (TrigFlow and rectified-flow), dCM, DMD and the
fake-score denoising critic.

Parity with train/wan/rcm/models/t2v_model_distill_rcm.py:
* ``_student_scm_step`` (:548-629): teacher F with CFG, tangents t_x = cos sin F_teacher, t_t = cos sin,
  student JVP (``student_F_withT`` :458-512, here ``student_F_with_tangent``), target
  g = -cos sqrt(1 - r^2 sin^2)(F_sg - F_teacher) - (r cos sin x_t + t_F), NaN masks, per-sample
  normalisation g / (||g|| + 0.1), loss ||F - F_sg - g||^2 summed, times ``loss_scale``;
  ``fd_type`` 1 / 2 finite-difference variants;
* ``_student_rf_scm_step`` (:631-684), ``_student_dcm_step`` (:686-735), ``_student_dmd_step`` (:737-773),
  ``training_step_critic`` (:775-795).
"""
from __future__ import annotations

import math

import numpy as np
import torch

from ..algorithms import LogNormal, rf_to_trig_time, shift_rf_time
from ..models.wan_jvp import wan_forward_jvp


def _t5(t):
    return t.reshape(-1, 1, 1, 1, 1)


def _uncond(batch):
    ctx = batch.get("neg_context")
    return ctx if ctx is not None else torch.zeros_like(batch["context"])


def teacher_F(m, xt, t, ctx, unctx):
    cfg = m.cfg
    with torch.no_grad():
        x0 = m.denoise(m.net_teacher, xt, t, ctx)
        F_ = (torch.cos(_t5(t)) * xt - x0) / torch.sin(_t5(t))
        if cfg.teacher_guidance > 1.0:
            x0u = m.denoise(m.net_teacher, xt, t, unctx)
            Fu = (torch.cos(_t5(t)) * xt - x0u) / torch.sin(_t5(t))
            F_ = Fu + cfg.teacher_guidance * (F_ - Fu)
    return F_.float()


def student_F(m, xt, t, ctx):
    x0 = m.denoise(m.net, xt, t, ctx)
    return (torch.cos(_t5(t)) * xt - x0) / torch.sin(_t5(t))


@torch.no_grad()
def student_F_with_tangent(m, xt, t_xt, t, t_t, ctx):
    """(F, t_F) of the student in TrigFlow parameterisation along (t_xt, t_t)."""
    t5, tt5 = _t5(t).double(), _t5(t_t).double()
    (c_skip, c_out, c_in, c_noise), (tc_skip, tc_out, tc_in, tc_noise) = torch.func.jvp(m.scaling, (t5,), (tt5,))
    x_in = xt * c_in
    tx_in = t_xt * c_in + xt * tc_in
    out, tout = wan_forward_jvp(m.net, x_in.to(m.dtype), tx_in.to(m.dtype), c_noise.reshape(-1, 1).to(m.dtype).float(),
                                tc_noise.reshape(-1, 1).to(m.dtype).float(), ctx)

    def proc(xt_, o, cs, co, tm):
        x0 = cs * xt_ + co * o
        return (torch.cos(tm) * xt_ - x0) / torch.sin(tm)

    F_, tF = torch.func.jvp(proc, (xt.double(), out.double(), c_skip, c_out, t5),
                            (t_xt.double(), tout.double(), tc_skip, tc_out, tt5))
    return F_.float(), tF.float()


def scm_loss(m, batch, it):
    """Per-sample sCM loss (TrigFlow parameterisation); backward is left to the caller."""
    cfg = m.cfg
    x0, ctx = batch["latents"], batch["context"]
    B = x0.shape[0]
    pG = LogNormal(*cfg.p_G_lognormal)
    t = rf_to_trig_time(pG((B, 1), device=m.device, dtype=torch.float64).clamp(0, 1))
    eps = torch.randn(x0.shape, device=m.device)
    c, s = torch.cos(_t5(t)), torch.sin(_t5(t))
    xt = (x0 * c + eps * s).float()
    Ft = teacher_F(m, xt, t, ctx, _uncond(batch))
    t_xt = (c * s * Ft).float()
    t_t = (c * s).reshape(B, 1)
    with torch.no_grad():
        if cfg.fd_type == 1:
            Fp, tF = student_F_with_tangent(m, xt, t_xt, t, 0 * t_t, ctx)
            h = cfg.fd_size
            Fm = student_F(m, xt, t - h, ctx)
            tF = tF + c * s * (np.cos(h) * Fp - Fm) / np.sin(h)
        elif cfg.fd_type == 2:
            h = cfg.fd_size
            Fp = student_F(m, xt, t, ctx)
            x2 = np.cos(h) * xt - np.sin(h) * Ft
            tF = c * s * (np.cos(h) * Fp - student_F(m, x2, t - h, ctx)) / np.sin(h)
        else:
            _, tF = student_F_with_tangent(m, xt, t_xt, t, t_t, ctx)
    Fth = student_F(m, xt, t, ctx).float()
    Fsg = Fth.detach().clone()
    r = 1.0 if cfg.tangent_warmup == 0 else min(1.0, it / cfg.tangent_warmup)
    g = -c * torch.sqrt(1 - r ** 2 * s ** 2) * (Fsg - Ft) - (r * c * s * xt + tF)
    bad = (torch.isnan(g).flatten(1).any(1) | torch.isnan(Fth).flatten(1).any(1)).view(B, 1, 1, 1, 1).expand_as(g)
    g = torch.where(bad, torch.zeros_like(g), g)
    Fth = torch.where(bad, torch.zeros_like(Fth), Fth)
    Fsg = torch.where(bad, torch.zeros_like(Fsg), Fsg)
    g = g.double() / (g.double().norm(p=2, dim=(1, 2, 3, 4), keepdim=True) + 0.1)
    return cfg.loss_scale * ((Fth - Fsg - g) ** 2).sum(dim=(1, 2, 3, 4))


def rf_scm_loss(m, batch, it):
    """Per-sample sCM loss in the rectified-flow parameterisation."""
    cfg = m.cfg
    x0, ctx = batch["latents"], batch["context"]
    B, _, T = x0.shape[:3]
    pG = LogNormal(*cfg.p_G_lognormal)
    tr = pG((B, 1), device=m.device, dtype=torch.float64).clamp(0, 1)
    eps = torch.randn(x0.shape, device=m.device)
    t5 = _t5(tr)
    xt = ((1 - t5) * x0 + t5 * eps).float()
    k = cfg.rectified_flow_t_scaling_factor

    def vel(net, x, ts):
        return net(x.to(m.dtype), (ts * k).to(m.dtype).float(), ctx).float()

    with torch.no_grad():
        vt = vel(m.net_teacher, xt, tr)
        if cfg.teacher_guidance > 1.0:
            vu = m.net_teacher(xt.to(m.dtype), (tr * k).to(m.dtype).float(), _uncond(batch)).float()
            vt = vu + cfg.teacher_guidance * (vt - vu)
        _, tv = wan_forward_jvp(m.net, xt.to(m.dtype), vt.to(m.dtype), (tr * k).to(m.dtype).float(),
                                torch.full_like(tr, k).float(), ctx)
    vth = vel(m.net, xt, tr)
    vsg = vth.detach().clone()
    r = 1.0 if cfg.tangent_warmup == 0 else min(1.0, it / cfg.tangent_warmup)
    g = -(vsg - vt) - r * t5.float() * tv.float()
    bad = (torch.isnan(g).flatten(1).any(1) | torch.isnan(vth).flatten(1).any(1)).view(B, 1, 1, 1, 1).expand_as(g)
    g = torch.where(bad, torch.zeros_like(g), g)
    vth = torch.where(bad, torch.zeros_like(vth), vth)
    vsg = torch.where(bad, torch.zeros_like(vsg), vsg)
    g = g.double() / (g.double().norm(p=2, dim=(1, 2, 3, 4), keepdim=True) + 0.1)
    return cfg.loss_scale * ((vth - vsg - g) ** 2).sum(dim=(1, 2, 3, 4))


def dcm_loss(m, batch, it):
    cfg = m.cfg
    x0, ctx = batch["latents"], batch["context"]
    B = x0.shape[0]
    eps = torch.randn(x0.shape, device=m.device)
    du = 1.0 / cfg.dcm_total_steps
    u = torch.rand(B, 1, device=m.device, dtype=torch.float64) * (1.0 - cfg.dcm_skipping_interval_steps * du)
    ts = [rf_to_trig_time(shift_rf_time(1.0 - (u + k * du), cfg.dcm_timestep_shift))
          for k in range(cfg.dcm_skipping_interval_steps + 1)]
    xt = (torch.cos(_t5(ts[0])) * x0 + torch.sin(_t5(ts[0])) * eps).float()
    x0p = m.denoise(m.net, xt, ts[0], ctx)
    with torch.no_grad():
        xk = xt
        for k in range(cfg.dcm_skipping_interval_steps):
            Ft = teacher_F(m, xk, ts[k], ctx, _uncond(batch))
            xk = (xk - _t5(ts[k] - ts[k + 1]) * Ft).float()
        tgt = m.denoise(m.net, xk, ts[-1], ctx)
    return cfg.loss_scale * ((x0p - tgt) ** 2).sum(dim=(1, 2, 3, 4))


def student_step_with_cm(m, batch, it):
    """Student phase of the rCM recipe: consistency loss, then the distribution-matching term (DMAD
    critic or DMD), one optimiser step for both."""
    cfg = m.cfg
    m.net.train()
    if cfg.cm_type == "dcm":
        lcm = dcm_loss(m, batch, it)
    elif cfg.use_rf_scm:
        lcm = rf_scm_loss(m, batch, it)
    else:
        lcm = scm_loss(m, batch, it)
    lcm.sum().backward()
    if it < cfg.tangent_warmup:
        m.sync_student.sync()
        m.opt_student.step()
        m.opt_student.zero_grad()
        return {"cm_loss": lcm.detach().mean()}
    out = m.student_step(batch, it) if cfg.critic_mode == "dmad" else student_dmd_step(m, batch, it, True)
    out["cm_loss"] = lcm.detach().mean()
    return out


def student_dmd_step(m, batch, it, do_step):
    cfg = m.cfg
    x0, ctx = batch["latents"], batch["context"]
    n_sim = m.effective_iteration(it) % cfg.max_simulation_steps_fake + 1
    G = m.backward_simulation(ctx, x0.shape, n_sim, with_grad=True)
    D = m.draw_time_D(x0.shape[0])
    xt = m._noise(G, D)
    with torch.no_grad():
        x_fake = m.denoise(m.net_fake_score, xt, D, ctx)
        x_teach = m.denoise(m.net_teacher, xt, D, ctx)
        if cfg.teacher_guidance > 1.0:
            xu = m.denoise(m.net_teacher, xt, D, _uncond(batch))
            x_teach = xu + cfg.teacher_guidance * (x_teach - xu)
        wf = (G.double() - x_teach.double()).abs().mean(dim=[1, 2, 3, 4], keepdim=True).clip(min=1e-5)
    grad = (x_fake.double() - x_teach.double()) / wf
    loss = (G.double() - (G.double() - grad).detach()) ** 2
    loss[torch.isnan(loss).flatten(1).any(1)] = 0
    loss = cfg.loss_scale_dmd * loss.sum(dim=(1, 2, 3, 4))
    loss.sum().backward()
    if do_step:
        m.sync_student.sync()
        beta = m.ema_beta(m.effective_iteration(it)) if cfg.ema_enabled else None
        m.opt_student.step(ema_beta=beta)
        m.opt_student.zero_grad()
    return {"dmd_loss": loss.detach().mean(), "n_sim": n_sim}


def critic_denoise_step(m, batch, it):
    """rCM's fake-score update: denoising loss on the student's samples, weighted by 1/sin^2."""
    cfg = m.cfg
    x0, ctx = batch["latents"], batch["context"]
    n_sim = m.effective_iteration_fake(it) % cfg.max_simulation_steps_fake + 1
    with torch.no_grad():
        G = m.backward_simulation(ctx, x0.shape, n_sim, with_grad=False)
    D = m.draw_time_D(x0.shape[0])
    xt = m._noise(G, D)
    x_fake = m.denoise(m.net_fake_score, xt, D, ctx)
    loss = ((G - x_fake) ** 2 / torch.sin(_t5(D)) ** 2).sum(dim=(1, 2, 3, 4))
    loss.sum().backward()
    m.sync_critic.sync()
    m.opt_critic.step()
    m.opt_critic.zero_grad()
    return {"critic_denoise_loss": loss.detach().mean(), "n_sim": n_sim}
