"""Calibration statistics of the recurrent update (stepquant/core.py:18-39).

``row_impact`` -- the squared transported read [D (q - beta k (k^T q))]^2 of
each key row (core.py:18-24); ``impact_factors`` -- the per-row weights
w = exp(gamma/2 (log omega - mean log omega)) (core.py:27-29);
``lifetime_weight`` -- sum_{t < horizon} retention^(2t) as a stable geometric
sum (core.py:32-39).  Host or device tensors alike.
"""
import torch


def row_impact(q, k, log_decay, beta):
    q, k = q.float(), k.float()
    decay = log_decay.float().exp()
    if decay.ndim == q.ndim - 1:
        decay = decay.unsqueeze(-1)
    return (decay * (q - beta.float().unsqueeze(-1) * k * (k * q).sum(-1, keepdim=True))).square()


def impact_factors(omega, gamma=0.25, floor=1e-20):
    log_w = omega.double().clamp_min(floor).log() * (gamma / 2)
    return (log_w - log_w.mean(-1, keepdim=True)).exp().float()


def lifetime_weight(mean_log_decay, horizon=2048):
    if horizon < 1 or torch.isnan(mean_log_decay).any() or (mean_log_decay > 0).any():
        raise ValueError("horizon must be positive and mean log retention must be <= 0")
    x = 2 * mean_log_decay.double()
    denominator = torch.where(x == 0, torch.full_like(x, -1), x)  # x = 0 (retention one) is the limit below
    result = torch.expm1(horizon * denominator) / torch.expm1(denominator)
    return torch.where(x == 0, torch.full_like(result, horizon), result)
