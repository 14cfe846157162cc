"""DMAD: Distribution Matching as Adversarial Distillation.

The critic shares one backbone between two binary heads:
  real head    d_real    : real data (T) vs student samples (G)
  teacher head d_teacher : teacher samples (Q) vs student samples (G)
Critic loss     softplus(-d_real(T)) + softplus(d_real(G)) + softplus(-d_teacher(Q)) + softplus(d_teacher(G))
Generator loss  -d_real(G) - w_gap * d_teacher(G)
``w_gap`` reweights the teacher term per noise band: an online EMA of the gap
E[d_real(T)] - E[d_real(Q)] per band becomes sigmoid((median - gap_band) / tau),
normalised by the mean band weight.

Parity (the three reference copies of these components):
  heads   train/wan/rcm/models/t2v_model_distill_dmad.py:36-50,
          train/h3/lightx2v_train/trainers/dmd/minimax_h3_dmad_trainer.py:51-65
  losses  t2v_model_distill_dmad.py:399-469, minimax_h3_dmad_trainer.py:332-378,
          train/image/main/edm/edm_guidance.py:191-267
  gap     t2v_model_distill_dmad.py:356-395 (all-reduced, bands = CDF deciles of p_D),
          minimax_h3_dmad_trainer.py:305-328 (per rank, bias-corrected, count-based readiness),
          edm_guidance.py:154-187 (all-reduced, bands = Karras index // 100, weighted-mean normalisation)
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

NUM_GAP_BANDS = 10


class CriticHeads(nn.Module):
    """Two per-token Linear-SiLU-Linear heads (fp32), mean-pooled by the caller.

    ``rms_input``: normalise the tokens with a non-affine RMSNorm first (the H3 variant,
    whose residual stream grows with depth)."""

    def __init__(self, dim: int, rms_input: bool = False, eps: float = 1e-5):
        super().__init__()
        self.rms_input, self.eps = rms_input, eps
        self.real = nn.Sequential(nn.Linear(dim, dim), nn.SiLU(), nn.Linear(dim, 1))
        self.teacher = nn.Sequential(nn.Linear(dim, dim), nn.SiLU(), nn.Linear(dim, 1))

    def forward(self, tokens):
        if self.rms_input:
            tokens = tokens * torch.rsqrt(tokens.pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return self.real(tokens), self.teacher(tokens)

    def pooled(self, tokens):
        """tokens [B, L, D] -> (d_real [B], d_teacher [B]) mean over tokens (fp32)."""
        r, t = self(tokens.float())
        return r.mean(dim=1).squeeze(-1), t.mean(dim=1).squeeze(-1)


def critic_bce_loss(d_real_T, d_real_G, d_teacher_Q, d_teacher_G):
    """Per-sample softplus BCE of both heads (T, Q labelled 1; G labelled 0)."""
    return F.softplus(-d_teacher_Q) + F.softplus(d_teacher_G) + F.softplus(-d_real_T) + F.softplus(d_real_G)


def generator_linear_loss(d_real_G, d_teacher_G, w_gap=None, E_w=1.0):
    """Per-sample linear logit loss -d_real(G) - (w/E_w) d_teacher(G)."""
    teacher_term = -d_teacher_G
    if w_gap is not None:
        teacher_term = teacher_term * w_gap / E_w
    return teacher_term - d_real_G


def critic_accuracies(d_real_T, d_real_G, d_teacher_Q, d_teacher_G):
    return {
        "dmad_acc_q": (d_teacher_Q > 0).float().mean(),
        "dmad_acc_t": (d_real_T > 0).float().mean(),
        "dmad_acc_g": 0.5 * ((d_real_G < 0).float().mean() + (d_teacher_G < 0).float().mean()),
    }


class GapRouter(nn.Module):
    """Online per-band gap EMA and the teacher-term weights derived from it.

    mode="allreduce"  (Wan / EDM): band sums and counts are all-reduced over ranks; a band
        is ready after its first measurement; EMA without bias correction; weights engage
        once ``min_ready`` bands are ready; E_w = mean weight over ready bands (clamped at 1e-3).
    mode="local"      (H3): per-rank scalar updates; bias-corrected EMA; a band is ready after
        ``band_min_count`` updates; weights engage with ``min_ready`` ready bands and only for a
        ready band; E_w clamped at 1e-4.
    """

    def __init__(self, mode: str = "allreduce", tau: float = 2.0, beta: float = 0.99, min_ready: int = 5,
                 band_min_count: int = 10, enabled: bool = True, group=None):
        super().__init__()
        assert mode in ("allreduce", "local")
        self.mode, self.tau, self.beta = mode, tau, beta
        self.min_ready, self.band_min_count, self.enabled = min_ready, band_min_count, enabled
        self.group = group
        self.register_buffer("gap_ema", torch.zeros(NUM_GAP_BANDS))
        self.register_buffer("gap_ready", torch.zeros(NUM_GAP_BANDS))  # allreduce: 0/1 flags, local: counts

    # ------------------------------------------------------------------ updates
    @torch.no_grad()
    def update(self, d_real_T, d_real_Q, band_T, band_Q):
        """All-reduced per-band update (Wan / EDM).  d_*: [N] logits, band_*: [N] long in [0, 10)."""
        dev = self.gap_ema.device
        bt, bq = band_T.reshape(-1).to(dev).long(), band_Q.reshape(-1).to(dev).long()
        sT = torch.zeros(NUM_GAP_BANDS, device=dev)
        cT = torch.zeros(NUM_GAP_BANDS, device=dev)
        sQ = torch.zeros(NUM_GAP_BANDS, device=dev)
        cQ = torch.zeros(NUM_GAP_BANDS, device=dev)
        sT.scatter_add_(0, bt, d_real_T.reshape(-1).float().to(dev))
        cT.scatter_add_(0, bt, torch.ones_like(bt, dtype=torch.float32))
        sQ.scatter_add_(0, bq, d_real_Q.reshape(-1).float().to(dev))
        cQ.scatter_add_(0, bq, torch.ones_like(bq, dtype=torch.float32))
        if dist.is_available() and dist.is_initialized():
            packed = torch.stack([sT, cT, sQ, cQ])
            dist.all_reduce(packed, op=dist.ReduceOp.SUM, group=self.group)
            sT, cT, sQ, cQ = packed.unbind(0)
        valid = (cT > 0) & (cQ > 0)
        gap_now = sT / cT.clamp(min=1) - sQ / cQ.clamp(min=1)
        fresh = valid & (self.gap_ready > 0)
        upd = torch.where(fresh, self.beta * self.gap_ema + (1 - self.beta) * gap_now, gap_now)
        self.gap_ema.copy_(torch.where(valid, upd, self.gap_ema))
        self.gap_ready.copy_(torch.where(valid, torch.ones_like(self.gap_ready), self.gap_ready))

    @torch.no_grad()
    def update_local(self, band: int, d_real_T, d_real_Q):
        """Per-rank scalar-band update (H3)."""
        g = (d_real_T.detach().float().mean() - d_real_Q.detach().float().mean()).to(self.gap_ema.device)
        self.gap_ema[band] = self.beta * self.gap_ema[band] + (1.0 - self.beta) * g
        self.gap_ready[band] += 1

    # ------------------------------------------------------------------ weights
    def _corrected(self):
        if self.mode == "local":
            return self.gap_ema / (1.0 - self.beta ** self.gap_ready.clamp(min=1.0))
        return self.gap_ema

    def ready_mask(self):
        if self.mode == "local":
            return self.gap_ready >= self.band_min_count
        return self.gap_ready > 0

    @torch.no_grad()
    def weights(self, bands):
        """(w [N] or None, E_w): per-sample weights for the given bands, None until enough bands are ready."""
        if not self.enabled:
            return None, 1.0
        ready = self.ready_mask()
        if int(ready.sum()) < self.min_ready:
            return None, 1.0
        corr = self._corrected()
        center = float(corr[ready].median())
        w_band = torch.sigmoid((center - corr) / self.tau)
        clamp = 1e-4 if self.mode == "local" else 1e-3
        E_w = float(w_band[ready].mean().clamp(min=clamp))
        bands = bands.reshape(-1).to(w_band.device).long()
        w = w_band[bands]
        if self.mode == "local":
            w = torch.where(ready[bands], w, torch.ones_like(w))
            E_w = torch.where(ready[bands], torch.full_like(w, E_w), torch.ones_like(w))
        return w, E_w

    def median(self):
        ready = self.ready_mask()
        return float(self._corrected()[ready].median()) if bool(ready.any()) else 0.0


def band_of_cdf(u):
    """Noise band = CDF decile of the time draw (equally populated bands)."""
    return (u * NUM_GAP_BANDS).long().clamp(0, NUM_GAP_BANDS - 1)
