"""Per-batch writeback budgets for STEPQuant@6 (stepquant/kernels/profiles.py:16-28).

Selects the background SM budget and chunk size by architecture and captured
batch tier (32, 64, 128, 256, 512).  The budgets here are for a 148-SM B200:
the reference's A800 (108-SM) budgets scaled by 148/108 and rounded to the
8-SM granularity of green-context splits.
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class WritebackProfile:
    sms: int
    chunk: int
    foreground_priority: bool = True


_GDN_SMS = {32: 40, 64: 32, 128: 88, 256: 112, 512: 112}
_GDN_CHUNK = {32: 64, 64: 64, 128: 128, 256: 256, 512: 64}
_KDA_SMS = {32: 40, 64: 40, 128: 40, 256: 40, 512: 64}
_KDA_CHUNK = {32: 64, 64: 64, 128: 128, 256: 256, 512: 128}


def stepquant6_profile(architecture, batch):
    if architecture not in ("gdn", "kda"):
        raise ValueError("architecture must be gdn or kda")
    if not isinstance(batch, int) or isinstance(batch, bool) or not 1 <= batch <= 512:
        raise ValueError("batch must be an integer in 1..512")
    tier = next(n for n in (32, 64, 128, 256, 512) if batch <= n)
    if architecture == "gdn":
        return WritebackProfile(_GDN_SMS[tier], _GDN_CHUNK[tier])
    return WritebackProfile(_KDA_SMS[tier], _KDA_CHUNK[tier])
