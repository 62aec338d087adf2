"""Offline calibration of a STEPQuant plan (stepquant/calibration.py:9-143), with
the candidate distortions measured on the GPU.

``LayerStatistics`` accumulates, per recurrent layer, the mean row impact
omega, the mean log retention and a reservoir of state snapshots
(reference calibration.py:9-44).  ``calibrate`` turns them into per-layer plans under a
nominal bit budget with the reference's procedure (calibration.py:76-143): for
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


class _Reservoir:
    """A uniform sample of at most ``capacity`` items from a stream (reservoir
    sampling): the n-th item offered replaces a random slot j < capacity with
    j drawn from [0, n) by a generator seeded 0, so the same stream keeps the
    same items as the reference calibrator."""

    def __init__(self, capacity):
        self.capacity = capacity
        self.items = []
        self.offered = 0
        self.generator = torch.Generator().manual_seed(0)

    def offer(self, make):
        self.offered += 1
        if len(self.items) < self.capacity:
            self.items.append(make())
            return
        slot = int(torch.randint(self.offered, (), generator=self.generator))
        if slot < self.capacity:
            self.items[slot] = make()


class LayerStatistics:
    """Per-layer calibration statistics: the running sums of the row impact
    omega and of the log retention (double, over every request of every
    update), and a reservoir of state snapshots taken every ``sample_every``-th
    update (reference calibration.py:9-44)."""

    def __init__(self, architecture, sample_every=8, max_snapshots=64):
        self.architecture = architecture
        self.sample_every = sample_every
        self.tokens = 0
        self.updates = 0
        self.sums = {}
        self.reservoir = _Reservoir(max_snapshots)

    def _accumulate(self, key, value):
        value = value.double().sum(0).cpu()
        self.sums[key] = value if key not in self.sums else self.sums[key] + value

    def observe(self, q, k, v, log_decay, beta, state):
        """One update: inputs [B, H, K] (log_decay [B, H] GDN, [B, H, K] KDA), states [B, H, K, V]."""
        self._accumulate("omega", row_impact(q, k, log_decay, beta))
        self._accumulate("log_decay", log_decay)
        self.tokens += q.shape[0]
        self.updates += 1
        if self.updates % self.sample_every == 0:
            for sample in state:
                self.reservoir.offer(lambda: sample.float().cpu().clone())

    def export(self):
        if not self.reservoir.items:
            raise ValueError("no state samples collected; increase calibration tokens or lower sample_every")
        return dict(architecture=self.architecture, omega=self.sums["omega"] / self.tokens,
                    log_decay=self.sums["log_decay"] / self.tokens, snapshots=torch.stack(self.reservoir.items),
                    tokens=self.tokens, sampled_states=self.reservoir.offered)


def _distortions(stat, candidates, impact, pivots, group_size, device):
    """Mean weighted squared error of each unit per candidate width, [units..., candidates], and
    the fp16 error of the same units (calibration.py:47-73)."""
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


class _Layer:
    """One layer's allocation units: impact factors, lifetime weights and, per
    candidate width, the lifetime-weighted distortion of every unit."""

    def __init__(self, stat, candidates, horizon, group, device):
        self.stat = stat
        self.impact = impact_factors(stat["omega"]).to(device)
        self.lifetime = lifetime_weight(stat["log_decay"], horizon)
        self.group, self.device, self.candidates = group, device, candidates
        no_pivots = torch.zeros_like(self.impact, dtype=torch.bool)
        distortion, fp = _distortions(stat, candidates, self.impact, no_pivots, group, device)
        self.unit_shape = distortion.shape[:-1]
        self.cost = self._weighted(distortion)
        self.fp_cost = (fp * self.lifetime).flatten()

    @property
    def units(self):
        return self.lifetime.numel()

    def _weighted(self, distortion):
        return (distortion * self.lifetime[..., None]).reshape(-1, len(self.candidates))

    def refit(self, pivots):
        """Costs measured again with ``pivots`` (this layer's unit mask) kept in fp16."""
        mask = pivots.reshape(self.impact.shape).to(self.device)
        return self._weighted(_distortions(self.stat, self.candidates, self.impact, mask, self.group,
                                           self.device)[0])

    def plan(self, widths, architecture):
        bits = widths.reshape(self.unit_shape)
        if architecture == "gdn":  # one width per head, repeated over its key rows
            bits = bits[:, None].expand(self.impact.shape).clone()
        entry = asdict(QuantizationPlan(architecture, bits.cpu(), self.impact.cpu(), self.group))
        entry.pop("extended_widths")  # the reference's plan record: architecture, bits, impact, group size
        return entry


def _pivot_mask(architecture, cost, fp_cost, candidates, nominal_budget, count):
    """The ``count`` units with the largest residual risk: under the first
    allocation for GDN heads, the 8-bit over fp16 excess for KDA rows."""
    if architecture == "gdn":
        first = allocate(cost, candidates, nominal_budget, architecture)
        risk = cost.gather(1, torch.searchsorted(torch.tensor(candidates), first)[:, None]).flatten()
    else:
        risk = cost[:, -1] - fp_cost
    mask = torch.zeros(len(cost), dtype=torch.bool)
    mask[torch.argsort(risk, descending=True, stable=True)[:count]] = True
    return mask


def calibrate(statistics, nominal_bits=6, pivots=None, horizon=2048, value_group_size=32, device="cuda"):
    """Plans for every layer under one global budget (reference calibration.py:76-143);
    a fp16 pivot counts as 8 bits of the nominal budget.

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
    if any(stat["architecture"] != architecture for stat in statistics.values()):
        raise ValueError("one architecture per calibration artifact")
    candidates = [2, 4, 6, 8] if nominal_bits == 4 else [4, 6, 8]
    layers = [_Layer(statistics[name], candidates, horizon, value_group_size, device) for name in names]
    bounds = torch.tensor([0] + [layer.units for layer in layers]).cumsum(0).tolist()
    cost = torch.cat([layer.cost for layer in layers])
    units = len(cost)
    if pivots is None:
        pivots = 32 if architecture == "gdn" else 512
    if not 0 <= pivots <= units:
        raise ValueError(f"pivot count {pivots} exceeds {units} units; set --pivots for small models")
    integer_budget = nominal_bits * units - 8 * pivots
    if integer_budget < (units - pivots) * min(candidates):
        raise ValueError("too many pivots for nominal pre-pivot budget")
    fp_cost = torch.cat([layer.fp_cost for layer in layers])
    pivot = _pivot_mask(architecture, cost, fp_cost, candidates, nominal_bits * units, pivots)
    if architecture == "kda" and pivots:
        cost = torch.cat([layer.refit(pivot[lo:hi]) for layer, lo, hi in zip(layers, bounds, bounds[1:])])
    widths = torch.full((units,), 16, dtype=torch.long)
    widths[~pivot] = allocate(cost[~pivot], candidates, integer_budget, architecture)
    plans = {name: layer.plan(widths[lo:hi], architecture)
             for name, layer, lo, hi in zip(names, layers, bounds, bounds[1:])}
    return dict(format_version=2, plans=plans,
                settings=dict(nominal_bits=nominal_bits, pivots=pivots, horizon=horizon,
                              value_group_size=value_group_size, candidates=candidates,
                              integer_budget=integer_budget, integer_bits_used=int(widths[~pivot].sum()),
                              calibration_tokens={name: statistics[name]["tokens"] for name in names}))
