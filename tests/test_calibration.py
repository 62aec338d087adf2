"""Calibration (stepquant/calibration.py, allocation.py) against golden vectors
of the reference (tests/golden/calibration.npz, made by make_golden.py).

CPU: the allocation solvers reproduce the reference's assignments on seeded
cost tables; ``LayerStatistics`` replaying the seeded observe() stream exports
exactly the reference's statistics.  GPU: ``calibrate`` on those statistics,
with its distortions from the device fit_state, returns the reference's plans.
"""
import importlib.util
import os

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = np.load(os.path.join(HERE, "golden", "calibration.npz"))


def _make_golden():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(HERE, "golden", "make_golden.py"))
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _statistics(arch, layers):
    stats = {}
    for layer in range(layers):
        tokens, sampled = (int(x) for x in GOLDEN[f"{arch}_{layer}_counts"])
        stats[f"model.layers.{3 * layer}.mixer"] = dict(
            architecture=arch, omega=torch.from_numpy(GOLDEN[f"{arch}_{layer}_omega"]),
            log_decay=torch.from_numpy(GOLDEN[f"{arch}_{layer}_log_decay"]),
            snapshots=torch.from_numpy(GOLDEN[f"{arch}_{layer}_snapshots"]), tokens=tokens, sampled_states=sampled)
    return stats


def test_allocation_solvers_match_reference():
    from stepquant_b200.allocation import allocate_dp, allocate_lagrangian
    for name, fn, candidates in (("dp", allocate_dp, [4, 6, 8]), ("lagrangian", allocate_lagrangian, [2, 4, 6, 8])):
        got = fn(GOLDEN[f"alloc_{name}_cost"], candidates, int(GOLDEN[f"alloc_{name}_budget"]))
        np.testing.assert_array_equal(got.numpy(), GOLDEN[f"alloc_{name}_result"])
        assert got.sum() <= int(GOLDEN[f"alloc_{name}_budget"])


def test_allocation_rejects_infeasible_and_nonfinite():
    from stepquant_b200.allocation import allocate, allocate_dp, allocate_lagrangian
    with pytest.raises(ValueError):
        allocate_dp(np.ones((4, 3)), [4, 6, 8], 15)
    with pytest.raises(ValueError):
        allocate_lagrangian(np.ones((4, 2)), [2, 4], 7)
    with pytest.raises(ValueError):
        allocate(np.array([[1.0, np.nan]]), [4, 6], 10, "gdn")


def test_layer_statistics_export_matches_reference():
    from stepquant_b200.calibration import LayerStatistics
    golden = _make_golden()
    for arch, layers, heads, keys, values, _, _, seed in golden.CALIBRATION_CASES:
        for layer in range(layers):
            got = golden.observe_run(LayerStatistics, arch, heads, keys, values, seed + 100 * layer)
            for key in ("omega", "log_decay", "snapshots"):
                np.testing.assert_array_equal(got[key].numpy(), GOLDEN[f"{arch}_{layer}_{key}"])
            assert [got["tokens"], got["sampled_states"]] == GOLDEN[f"{arch}_{layer}_counts"].tolist()


def test_calibrate_rejects_cpu_and_bad_budgets():
    from stepquant_b200.calibration import calibrate
    stats = _statistics("gdn", 2)
    with pytest.raises(ValueError):
        calibrate(stats, device="cpu")
    with pytest.raises(ValueError):
        calibrate({}, device="cuda")
    with pytest.raises(ValueError):
        calibrate(stats, nominal_bits=5, device="cuda")


@pytest.mark.gpu
@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_calibrate_on_gpu_matches_reference_plans(arch):
    from stepquant_b200.calibration import calibrate
    golden = _make_golden()
    case = next(c for c in golden.CALIBRATION_CASES if c[0] == arch)
    _, layers, _, _, _, nominal, pivots, _ = case
    stats = _statistics(arch, layers)
    result = calibrate(stats, nominal_bits=nominal, pivots=pivots, horizon=256, value_group_size=8, device="cuda")
    assert result["format_version"] == 2
    for layer, name in enumerate(sorted(stats)):
        plan = result["plans"][name]
        np.testing.assert_array_equal(plan["bits"].numpy(), GOLDEN[f"{arch}_{layer}_bits"])
        np.testing.assert_array_equal(plan["impact"].numpy(), GOLDEN[f"{arch}_{layer}_impact"])
    st = result["settings"]
    assert [st["integer_budget"], st["integer_bits_used"]] == GOLDEN[f"{arch}_budget"].tolist()
