"""Teacher samplers for flow-matching models (velocity prediction, x_sigma = (1-sigma) x0 + sigma eps).

Parity: ``FlowEulerSampler`` (train/wan/rcm/samplers/euler.py) and ``FlowUniPCMultistepSampler``
(train/wan/rcm/samplers/unipc.py), both with the shifted grid ``shift*s / (1 + (shift-1)*s)`` over
``linspace(1, 0, n+1)[:-1]`` and timesteps ``1000*sigma``; used for teacher data (100-step Euler,
CFG 5, shift 3) and the teacher baseline.

UniPC is written from the published method (Zhao et al., "UniPC: A Unified Predictor-Corrector
Framework for Fast Sampling of Diffusion Models", NeurIPS 2023) in its data-prediction form:
with alpha = 1 - sigma, lambda = log(alpha / sigma) and h = lambda_t - lambda_s, the predictor is

    x_t = (sigma_t / sigma_s) x_s - alpha_t (e^{-h} - 1) m_s - alpha_t B(h) sum_k rho_k D_k

(D_k = (m_{s_k} - m_s) / r_k the scaled differences of earlier x0 predictions, r_k their
log-SNR offsets / h, rho solving the order conditions R rho = g(h)), and the corrector repeats the
update with the fresh prediction at t (UniC).  B(h) = e^{-h} - 1 ("bh2", the default) or -h ("bh1").
"""
from __future__ import annotations

import math

import torch


def shifted_sigmas(n: int, shift: float, sigma_max: float = 1.0, sigma_min: float = 0.0) -> torch.Tensor:
    s = torch.linspace(sigma_max, sigma_min, n + 1, dtype=torch.float64)[:-1]
    return shift * s / (1 + (shift - 1) * s)


class FlowEulerSampler:
    def __init__(self, num_train_timesteps: int = 1000, sigma_max: float = 1.0, sigma_min: float = 0.0):
        self.T, self.sigma_max, self.sigma_min = num_train_timesteps, sigma_max, sigma_min

    def set_timesteps(self, num_inference_steps: int = 100, shift: float = 3.0, device="cpu"):
        s = shifted_sigmas(num_inference_steps, shift, self.sigma_max, self.sigma_min)
        self.sigmas = s.to(device=device, dtype=torch.float32)
        self.timesteps = (s * self.T).to(device=device, dtype=torch.float32)

    def step(self, model_output, timestep, sample):
        i = int(torch.argmin((self.timesteps - timestep).abs()))
        s = self.sigmas[i]
        s_next = self.sigmas[i + 1] if i + 1 < len(self.sigmas) else 0.0
        return sample + model_output * (s_next - s)


class FlowUniPCSampler:
    def __init__(self, num_train_timesteps: int = 1000, solver_order: int = 2, solver_type: str = "bh2",
                 lower_order_final: bool = True, sigma_max: float = 1.0, sigma_min: float = 0.0):
        if solver_type not in ("bh1", "bh2"):
            raise ValueError(solver_type)
        self.T, self.order, self.kind, self.lower_final = num_train_timesteps, solver_order, solver_type, \
            lower_order_final
        self.sigma_max, self.sigma_min = sigma_max, sigma_min

    def set_timesteps(self, num_inference_steps: int = 50, shift: float = 3.0, device="cpu"):
        s = shifted_sigmas(num_inference_steps, shift, self.sigma_max, self.sigma_min)
        self.sig = torch.cat([s, torch.zeros(1, dtype=torch.float64)])  # float64 host copy for the coefficients
        self.sigmas = self.sig.to(device=device, dtype=torch.float32)
        self.timesteps = (s * self.T).to(device=device, dtype=torch.float32)
        self.n = num_inference_steps
        self.i = 0
        self.hist: list[torch.Tensor] = []      # x0 predictions, newest last
        self.hist_lam: list[float] = []
        self.last_sample = None

    @staticmethod
    def _lam(sig: float) -> float:
        if sig <= 0.0:
            return math.inf
        if sig >= 1.0:
            return -math.inf
        return math.log(1.0 - sig) - math.log(sig)

    def _coeffs(self, h: float, rks: list[float], corrector: bool):
        """rho for the order conditions (the last entry weighs the corrector's own difference)."""
        hh = -h
        if math.isinf(hh):
            phi1 = -1.0
        else:
            phi1 = math.expm1(hh)
        B = hh if self.kind == "bh1" else phi1
        order = len(rks)
        # first-order corrector and second-order predictor use the fixed weight 1/2 (also across the
        # infinite log-SNR step out of sigma = 1)
        if corrector and order == 1:
            return phi1, B, [0.5]
        if not corrector and order <= 2:
            return phi1, B, ([] if order == 1 else [0.5])
        if math.isinf(hh):
            return phi1, B, [1.0] * len(rks)
        R, g = [], []
        phik = phi1 / hh - 1.0
        fact = 1.0
        for k in range(1, order + 1):
            R.append([r ** (k - 1) for r in rks])
            g.append(phik * fact / B)
            fact *= k + 1
            phik = phik / hh - 1.0 / fact
        if not corrector:
            m = order - 1  # the predictor has no term at r = 1
            Rm = torch.tensor([row[:m] for row in R[:m]], dtype=torch.float64)
            return phi1, B, torch.linalg.solve(Rm, torch.tensor(g[:m], dtype=torch.float64)).tolist()
        return phi1, B, torch.linalg.solve(torch.tensor(R, dtype=torch.float64),
                                           torch.tensor(g, dtype=torch.float64)).tolist()

    def _update(self, x, m0, s_sig, t_sig, lam_s, olds, corrector_m=None):
        """One UniP (or UniC when ``corrector_m`` is the prediction at t) update from s to t."""
        lam_t = self._lam(t_sig)
        h = lam_t - lam_s
        rks, D = [], []
        for mi, lam_i in olds:
            r = (lam_i - lam_s) / h
            rks.append(r)
            D.append((mi - m0) / r)
        rks.append(1.0)
        phi1, B, rho = self._coeffs(h, rks, corrector_m is not None)
        alpha_t = 1.0 - t_sig
        out = (t_sig / s_sig) * x - alpha_t * phi1 * m0
        res = None
        for k, d in enumerate(D):
            term = rho[k] * d
            res = term if res is None else res + term
        if corrector_m is not None:
            term = rho[-1] * (corrector_m - m0)
            res = term if res is None else res + term
        if res is not None:
            out = out - alpha_t * B * res
        return out

    def step(self, model_output, timestep, sample):
        i = self.i
        sig = float(self.sig[i])
        m = sample - sig * model_output  # x0 prediction from the velocity
        if i > 0 and self.last_sample is not None:
            # corrector of the previous step with the fresh prediction at this sigma
            s_prev = float(self.sig[i - 1])
            m_prev, lam_prev = self.hist[-1], self.hist_lam[-1]
            olds = list(zip(self.hist[:-1][::-1], self.hist_lam[:-1][::-1]))[: self._order_c - 1]
            sample = self._update(self.last_sample, m_prev, s_prev, sig, lam_prev, olds, corrector_m=m)
        self.hist.append(m)
        self.hist_lam.append(self._lam(sig))
        self.hist = self.hist[-self.order:]
        self.hist_lam = self.hist_lam[-self.order:]
        order = min(self.order, self.n - i) if self.lower_final else self.order
        order = min(order, len(self.hist))
        self._order_c = order
        self.last_sample = sample
        olds = list(zip(self.hist[:-1][::-1], self.hist_lam[:-1][::-1]))[: order - 1]
        x_next = self._update(sample, m, sig, float(self.sig[i + 1]), self.hist_lam[-1], olds)
        self.i += 1
        return x_next


@torch.no_grad()
def sample_flow(velocity_fn, noise, num_steps: int = 100, shift: float = 3.0, sampler: str = "euler",
                guidance: float = 1.0, uncond_velocity_fn=None):
    """Integrate ``velocity_fn(x, t)`` (t = 1000*sigma) from sigma = 1 to 0 with classifier-free
    guidance ``v = v_u + g (v_c - v_u)`` when ``uncond_velocity_fn`` is given."""
    smp = FlowEulerSampler() if sampler == "euler" else FlowUniPCSampler()
    smp.set_timesteps(num_steps, shift, device=noise.device)
    x = noise
    for t in smp.timesteps:
        v = velocity_fn(x, t)
        if uncond_velocity_fn is not None and guidance != 1.0:
            vu = uncond_velocity_fn(x, t)
            v = vu + guidance * (v - vu)
        x = smp.step(v, t, x)
    return x
