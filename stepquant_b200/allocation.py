"""Bit allocation from frozen candidate distortions (stepquant/allocation.py:6-81).

``allocate_dp`` -- exact minimum total distortion under an integer bit budget
(one width per unit), a knapsack over the budget in unit order: for each unit
the candidates are tried in ascending width and a state improves only on a
strictly smaller cost; the answer is the first budget with the least cost,
traced back unit by unit (GDN heads).  ``allocate_lagrangian`` -- the widths
minimising cost + lambda * width for the smallest feasible lambda (80 bisection
steps), then the leftover bits spent on the upgrades of best gain per bit
(KDA rows).  Host code (numpy): the inputs are small cost tables.
"""
import heapq

import numpy as np
import torch


def allocate_dp(cost, candidates, budget):
    cost = np.asarray(cost, dtype=np.float64)
    widths = np.asarray(candidates, dtype=int)
    units, _ = cost.shape
    if budget < units * widths.min():
        raise ValueError("integer budget is infeasible")
    budget = min(int(budget), units * int(widths.max()))
    best = np.full(budget + 1, np.inf)
    best[0] = 0.0
    choice = np.full((units, budget + 1), -1, dtype=np.int8)
    for unit in range(units):
        step = np.full(budget + 1, np.inf)
        for j, width in enumerate(widths):
            candidate = best[:budget + 1 - width] + cost[unit, j]
            improves = candidate < step[width:]
            step[width:][improves] = candidate[improves]
            choice[unit, width:][improves] = j
        best = step
    spent = int(best.argmin())
    result = np.empty(units, dtype=np.int64)
    for unit in range(units - 1, -1, -1):
        j = choice[unit, spent]
        if j < 0:
            raise RuntimeError("allocation backtracking failed")
        result[unit] = widths[j]
        spent -= int(widths[j])
    return torch.from_numpy(result)


def allocate_lagrangian(cost, candidates, budget):
    cost = np.asarray(cost, dtype=np.float64)
    widths = np.asarray(candidates, dtype=int)
    units = len(cost)
    if budget < units * widths.min():
        raise ValueError("integer budget is infeasible")
    if units == 0:
        return torch.empty(0, dtype=torch.long)

    def cheapest(lam):
        return np.argmin(cost + lam * widths, axis=1)

    pick = cheapest(0.0)
    if widths[pick].sum() <= budget:
        return torch.from_numpy(widths[pick].copy())
    lo, hi = 0.0, max(float(np.ptp(cost, axis=1).max()), 1e-30)
    for _ in range(80):
        lam = (lo + hi) / 2
        trial = cheapest(lam)
        if widths[trial].sum() > budget:
            lo = lam
        else:
            hi, pick = lam, trial
    left = int(budget - widths[pick].sum())
    # Every improving upgrade is a candidate (the cost curve need not be monotone).
    queue = []

    def offer(unit):
        now = pick[unit]
        for up in range(now + 1, len(widths)):
            gain = cost[unit, now] - cost[unit, up]
            if gain > 0:
                heapq.heappush(queue, (-gain / (widths[up] - widths[now]), unit, now, up))

    for unit in range(units):
        offer(unit)
    while queue and left:
        _, unit, now, up = heapq.heappop(queue)
        if now != pick[unit] or widths[up] - widths[now] > left:
            continue
        left -= int(widths[up] - widths[now])
        pick[unit] = up
        offer(unit)
    return torch.from_numpy(widths[pick].copy())


def allocate(cost, candidates, budget, architecture):
    if not np.isfinite(np.asarray(cost)).all():
        raise ValueError("candidate distortion must be finite")
    return (allocate_dp if architecture == "gdn" else allocate_lagrangian)(cost, candidates, budget)
