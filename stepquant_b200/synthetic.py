"""Seeded synthetic workloads for the decode path (no datasets or checkpoints).

Distributions follow the benchmark configurations: q, k ~ N(0, 1) (the kernel
L2-normalises them, scale K^-1/2), v ~ N(0, 1) in bf16, raw gate a ~ N(0, 1)
with A_log ~ U(0, ln 16) and dt_bias = 0 (log decay = -exp(A_log) *
softplus(a)), beta logit b ~ N(0, 1).  Plans: per-head GDN widths from
{4, 6, 8} at 25/50/25 (KDA: per-row widths), optional fp16 pivot heads/rows,
and impact factors fitted from row-impact statistics of a warm-up run the way
the reference calibrator does (core.py:18-29 ``row_impact`` /
``impact_factors``, calibration.py:22-44 ``LayerStatistics.observe``).
"""
import math
from dataclasses import dataclass

import torch

from .core import impact_factors, row_impact  # noqa: F401  (re-exported for the benchmark)

from .quantization import QuantizationPlan


@dataclass
class DecodeInputs:
    q: torch.Tensor      # [B, HK, K] bf16
    k: torch.Tensor      # [B, HK, K] bf16
    v: torch.Tensor      # [B, H, V] bf16
    a: torch.Tensor      # [B, H] (GDN) or [B, H, K] (KDA) fp32 raw gate
    b: torch.Tensor      # [B, H] fp32 beta logits


def draw_inputs(batch, heads, qk_heads, keys, values, kda, generator, device="cuda", dtype=torch.bfloat16):
    q = torch.randn(batch, qk_heads, keys, generator=generator, device=device).to(dtype)
    k = torch.randn(batch, qk_heads, keys, generator=generator, device=device).to(dtype)
    v = torch.randn(batch, heads, values, generator=generator, device=device).to(dtype)
    a = torch.randn(batch, heads, keys, generator=generator, device=device) if kda else \
        torch.randn(batch, heads, generator=generator, device=device)
    b = torch.randn(batch, heads, generator=generator, device=device)
    return DecodeInputs(q, k, v, a, b)


def gate_parameters(heads, keys, kda, generator, device="cuda"):
    a_log = torch.rand(heads, generator=generator, device=device) * math.log(16)
    dt_bias = torch.zeros(heads * keys if kda else heads, device=device)
    return a_log, dt_bias


def prepared(inputs, heads, keys, kda, a_log, dt_bias):
    """q, k normalised and broadcast to value heads, log decay and beta (fp32)."""
    q = inputs.q.float()
    k = inputs.k.float()
    q = q * torch.rsqrt(q.square().sum(-1, keepdim=True) + 1e-6) * keys ** -0.5
    k = k * torch.rsqrt(k.square().sum(-1, keepdim=True) + 1e-6)
    rep = heads // q.shape[1]
    q, k = q.repeat_interleave(rep, 1), k.repeat_interleave(rep, 1)
    if kda:
        u = inputs.a + dt_bias.reshape(heads, keys)
        g = -a_log.exp()[:, None] * torch.nn.functional.softplus(u)
    else:
        g = -a_log.exp() * torch.nn.functional.softplus(inputs.a + dt_bias)
    return q, k, g, torch.sigmoid(inputs.b)




def gdn_widths(heads, generator, pivot_heads=0, two_bit_heads=0):
    """Per-head widths {4, 6, 8} at 25/50/25, permuted; the first ``pivot_heads`` of the permutation become fp16,
    the next ``two_bit_heads`` 2-bit (value groups of 32)."""
    counts = [heads // 4, heads - 2 * (heads // 4), heads // 4]
    widths = [4] * counts[0] + [6] * counts[1] + [8] * counts[2]
    perm = torch.randperm(heads, generator=generator).tolist()
    widths = [widths[i] for i in perm]
    for i in range(pivot_heads):
        widths[i] = 16
    for i in range(pivot_heads, pivot_heads + two_bit_heads):
        widths[i] = 2
    return torch.tensor(widths)


def kda_widths(heads, keys, generator, choices=(2, 4, 6), probs=(0.3, 0.5, 0.2), pivot_fraction=0.02):
    idx = torch.multinomial(torch.tensor(probs), heads * keys, True, generator=generator).reshape(heads, keys)
    bits = torch.tensor(choices)[idx]
    bits[torch.rand(heads, keys, generator=generator) < pivot_fraction] = 16
    return bits


def warm_state(step_fn, batch, heads, qk_heads, keys, values, kda, steps, generator, a_log, dt_bias, device="cuda"):
    """Run ``steps`` unquantized updates from zero; returns (state, omega [H, K]).

    ``step_fn(state, inputs)`` advances an fp32 state in place (the FP32 pool
    kernel in the benchmark).  omega is the mean row impact of the inputs.
    """
    state = torch.zeros(batch, heads, keys, values, device=device)
    omega = torch.zeros(heads, keys, device=device, dtype=torch.float64)
    for _ in range(steps):
        inputs = draw_inputs(batch, heads, qk_heads, keys, values, kda, generator, device)
        step_fn(state, inputs)
        q, k, g, beta = prepared(inputs, heads, keys, kda, a_log, dt_bias)
        omega += row_impact(q, k, g, beta).double().sum(0)
    return state, (omega / (steps * batch)).float()


def gdn_plan(bits_per_head, keys, impact, group=32):
    bits = bits_per_head[:, None].expand(len(bits_per_head), keys).clone()
    return QuantizationPlan("gdn", bits, impact, group)
