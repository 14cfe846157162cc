"""Distillation algorithms: DMAD critic/generator losses, gap routing, EMA,
noise-time distributions and the TrigFlow / rectified-flow conversions."""
from .timesteps import (LogNormal, UniformShift, rf_to_trig_time, trig_to_rf_time, shift_rf_time,
                        inverse_shift_rf_time, sigma_to_rf_time, rf_to_sigma, TrigFlowScaling)
from .dmad import (CriticHeads, GapRouter, critic_bce_loss, generator_linear_loss, NUM_GAP_BANDS)
from .ema import power_ema_beta, ema_exp_coefficient, PowerEMA, kimg_halflife_beta

__all__ = [
    "LogNormal", "UniformShift", "rf_to_trig_time", "trig_to_rf_time", "shift_rf_time", "inverse_shift_rf_time",
    "sigma_to_rf_time", "rf_to_sigma", "TrigFlowScaling", "CriticHeads", "GapRouter", "critic_bce_loss",
    "generator_linear_loss", "NUM_GAP_BANDS", "power_ema_beta", "ema_exp_coefficient", "PowerEMA",
    "kimg_halflife_beta",
]
