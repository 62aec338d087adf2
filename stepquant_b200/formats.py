"""State-format registry (the reference's ``stepquant.formats`` API, formats.py:28-44,85-101).

Formats are named records; ``stepquant4`` / ``stepquant6`` are the calibrated
packed formats (``PackedStatePool``).  The paper baselines run on the device
too: fp32 through ``Fp32StatePool`` (``sq_fp32_step``), sym_int*_g128 and
dsq_int* through ``FormatStatePool`` (the tile kernel with ``sq_plan.storage``
2 and 3).
"""
from dataclasses import asdict, dataclass
import re

import torch


@dataclass(frozen=True)
class StateFormat:
    name: str
    kind: str
    bits: int = 8
    group_size: int = 32
    group_axis: str = "v"

    @property
    def calibrated(self):
        return self.kind == "stepquant"

    def to_dict(self):
        return asdict(self)


def get_format(name):
    """formats.py:28-39."""
    if name in ("stepquant", "stepquant4", "stepquant6"):
        return StateFormat(name, "stepquant", 4 if name.endswith("4") else 6, 32)
    if name == "fp32":
        return StateFormat(name, "fp32", 32, 32)
    match = re.fullmatch(r"sym_int([468])_g128", name)
    if match:
        return StateFormat(name, "symmetric", int(match[1]), 128)
    match = re.fullmatch(r"dsq_int([46])", name)
    if match:
        return StateFormat(name, "dsq", int(match[1]), 128, group_axis="k")
    raise ValueError(f"unknown state format: {name}")


BASELINE_NAMES = ["fp32", "sym_int4_g128", "sym_int6_g128", "sym_int8_g128", "dsq_int4", "dsq_int6"]
FORMAT_NAMES = BASELINE_NAMES + ["stepquant4", "stepquant6"]


@dataclass
class FormatPlan:
    """Plan record of the baseline formats (formats.py:85-101)."""
    architecture: str
    bits: torch.Tensor
    impact: torch.Tensor
    value_group_size: int = 32

    def __post_init__(self):
        if self.architecture not in ("gdn", "kda") or self.bits.ndim != 2 or self.bits.shape != self.impact.shape:
            raise ValueError("invalid format plan shape/architecture")
        if not torch.isin(self.bits, torch.tensor([2, 4, 6, 8, 16, 32], device=self.bits.device)).all():
            raise ValueError("invalid state precision")
        if not torch.isfinite(self.impact).all() or (self.impact <= 0).any():
            raise ValueError("impact must be finite and positive")

    def to(self, device):
        return FormatPlan(self.architecture, self.bits.to(device), self.impact.to(device), self.value_group_size)
