"""Offline calibration of a STEPQuant plan (stepquant/calibration.py:9-143), with
the candidate distortions measured on the GPU.

``LayerStatistics`` accumulates, per recurrent layer, the mean row impact
omega, the mean log retention and a reservoir of state snapshots
(calibration.py:9-44).  ``calibrate`` turns them into per-layer plans under a
nominal bit budget with the reference's procedure (calibration.py:74-143): for
every candidate width the snapshots are quantized with ``fit_state`` and the
impact-weighted squared reconstruction error is averaged per allocation unit
(a GDN head, a KDA key row); units are weighted by their lifetime, fp16 pivots
are chosen by residual risk, and ``allocation.allocate`` distributes the
integer budget.  The distortions are the expensive part: here all snapshots of
a layer go through the device ``fit_state`` (``sq_fit_state``) as one batch per
candidate, instead of one CPU call per snapshot.  The result is the plan
artifact of ``stepquant.sglang`` (format_version 2).
"""
from dataclasses import asdict

import torch

from .allocation import allocate
from .core import impact_factors, lifetime_weight, row_impact
from .quantization import QuantizationPlan, fit_state


class LayerStatistics:
    def __init__(self, architecture, sample_every=8, max_snapshots=64):
        self.architecture = architecture
        self.sample_every = sample_every
        self.max_snapshots = max_snapshots
        self.count = 0
        self.updates = 0
        self.omega = None
        self.log_decay = None
        self.snapshots = []
        self.sample_count = 0
        self.rng = torch.Generator().manual_seed(0)

    def observe(self, q, k, v, log_decay, beta, state):
        """One update's inputs [B, H, K] (log_decay [B, H] GDN, [B, H, K] KDA) and its states [B, H, K, V]."""
        omega = row_impact(q, k, log_decay, beta).double().sum(0).cpu()
        decay = log_decay.double().sum(0).cpu()
        self.omega = omega if self.omega is None else self.omega + omega
        self.log_decay = decay if self.log_decay is None else self.log_decay + decay
        self.count += q.shape[0]
        self.updates += 1
        if self.updates % self.sample_every:
            return
        for sample in state:  # reservoir of max_snapshots states
            self.sample_count += 1
            if len(self.snapshots) < self.max_snapshots:
                self.snapshots.append(sample.float().cpu().clone())
            else:
                slot = torch.randint(self.sample_count, (), generator=self.rng).item()
                if slot < self.max_snapshots:
                    self.snapshots[slot] = sample.float().cpu().clone()

    def export(self):
        if not self.snapshots:
            raise ValueError("no state samples collected; increase calibration tokens or lower sample_every")
        return dict(architecture=self.architecture, omega=self.omega / self.count,
                    log_decay=self.log_decay / self.count, snapshots=torch.stack(self.snapshots),
                    tokens=self.count, sampled_states=self.sample_count)


def _distortions(stat, candidates, impact, pivots, group_size, device):
    """Mean weighted squared error of each unit per candidate width, [units..., candidates], and
    the fp16 error of the same units (calibration.py:47-71)."""
    architecture = stat["architecture"]
    x = stat["snapshots"].to(device=device, dtype=torch.float32)
    dims = (2, 3) if architecture == "gdn" else (3,)  # per snapshot: a head, or a key row
    weights = impact[None, :, :, None].square() if architecture == "gdn" else None

    def unit_means(error):
        if weights is not None:
            error = error * weights
        means = error.mean(dims).cpu().double()
        total = torch.zeros_like(means[0])
        for m in means:  # snapshot order, in double
            total = total + m
        return total / means.shape[0]

    losses = []
    for bit in candidates:
        bits = torch.full(impact.shape, bit, dtype=torch.long, device=device)
        bits[pivots] = 16
        plan = QuantizationPlan(architecture, bits, impact, group_size)
        losses.append(unit_means((fit_state(x, plan)[-1] - x).square()))
    # The fp16 error does not depend on the candidate.
    fp = unit_means((x.half().float() - x).square())
    return torch.stack(losses, -1), fp


def calibrate(statistics, nominal_bits=6, pivots=None, horizon=2048, value_group_size=32, device="cuda"):
    """Global allocation across layers; a fp16 pivot counts as 8 bits of the nominal budget.

    GDN: an exact DP over heads, pivots where the allocated residual risk is
    largest, then the DP again on the rest.  KDA: pivots where the fp16 gain
    over 8 bits (lifetime-weighted) is largest, distortions refitted without
    them, then the Lagrangian allocation over rows.
    """
    if torch.device(device).type != "cuda":
        raise ValueError("calibration measures its distortions on a CUDA device")
    if nominal_bits not in (4, 6) or not statistics:
        raise ValueError("provide statistics and nominal_bits=4 or 6")
    names = sorted(statistics)
    architecture = statistics[names[0]]["architecture"]
    if any(s["architecture"] != architecture for s in statistics.values()):
        raise ValueError("one architecture per calibration artifact")
    candidates = [2, 4, 6, 8] if nominal_bits == 4 else [4, 6, 8]
    info, costs, fps = {}, [], []
    for name in names:
        stat = statistics[name]
        w = impact_factors(stat["omega"]).to(device)
        d, fp = _distortions(stat, candidates, w, torch.zeros_like(w, dtype=torch.bool), value_group_size, device)
        lifetime = lifetime_weight(stat["log_decay"], horizon)
        info[name] = (w, lifetime, d.shape[:-1])
        costs.append((d * lifetime[..., None]).reshape(-1, len(candidates)))
        fps.append((fp * lifetime).flatten())
    cost, fp = torch.cat(costs), torch.cat(fps)
    units = len(cost)
    pivots = (32 if architecture == "gdn" else 512) if pivots is None else pivots
    if not 0 <= pivots <= units:
        raise ValueError(f"pivot count {pivots} exceeds {units} units; set --pivots for small models")
    integer_budget = nominal_bits * units - 8 * pivots
    if integer_budget < (units - pivots) * min(candidates):
        raise ValueError("too many pivots for nominal pre-pivot budget")
    if architecture == "gdn":
        first = allocate(cost, candidates, nominal_bits * units, architecture)
        risk = cost.gather(1, torch.searchsorted(torch.tensor(candidates), first)[:, None]).flatten()
    else:
        risk = cost[:, -1] - fp
    pivot_mask = torch.zeros(units, dtype=torch.bool)
    pivot_mask[torch.argsort(risk, descending=True, stable=True)[:pivots]] = True
    if architecture == "kda" and pivots:
        start, revised = 0, []
        for name in names:
            w, lifetime, _ = info[name]
            size = lifetime.numel()
            mask = pivot_mask[start:start + size].reshape(w.shape).to(device)
            d, _ = _distortions(statistics[name], candidates, w, mask, value_group_size, device)
            revised.append((d * lifetime[..., None]).reshape(-1, len(candidates)))
            start += size
        cost = torch.cat(revised)
    assignment = torch.full((units,), 16, dtype=torch.long)
    assignment[~pivot_mask] = allocate(cost[~pivot_mask], candidates, integer_budget, architecture)
    plans, start = {}, 0
    for name in names:
        w, lifetime, unit_shape = info[name]
        size = lifetime.numel()
        bits = assignment[start:start + size].reshape(unit_shape)
        if architecture == "gdn":
            bits = bits[:, None].expand(w.shape).clone()
        plans[name] = asdict(QuantizationPlan(architecture, bits.cpu(), w.cpu(), value_group_size))
        start += size
    return dict(format_version=2, plans=plans,
                settings=dict(nominal_bits=nominal_bits, pivots=pivots, horizon=horizon,
                              value_group_size=value_group_size, candidates=candidates,
                              integer_budget=integer_budget, integer_bits_used=int(assignment[~pivot_mask].sum()),
                              calibration_tokens={name: statistics[name]["tokens"] for name in names}))
