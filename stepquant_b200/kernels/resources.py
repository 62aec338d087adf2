"""Writeback streams with an SM budget (interface of stepquant/kernels/resources.py).

``writeback_resources(device, sm_budget)`` returns the stream the background
requantization runs on.  A budget of 0 is an ordinary stream on the whole
device.  A nonzero budget is served by the native library
(``sq_budget_stream``, csrc/sq_streams.cu): a stream of a CUDA green context
that owns at least that many SMs, so the writeback cannot take SMs from the
foreground decode; the persistent kernels size their grids to the SMs of the
stream they run on.  Results are cached per (device, budget) for the process,
as captured graphs keep referring to the stream.
"""
import ctypes
from dataclasses import dataclass

import torch

from .. import _native as N


@dataclass
class WritebackResources:
    stream: torch.cuda.Stream
    requested_sms: int
    actual_sms: int
    total_sms: int
    context: object = None     # the green context stays owned by the native library
    descriptor: object = None


_cache = {}


def _ordinal(device):
    device = torch.device(device)
    return torch.cuda.current_device() if device.index is None else device.index


def _budget_stream(ordinal, sm_budget):
    stream, actual, total = ctypes.c_void_p(), ctypes.c_int32(), ctypes.c_int32()
    code = N.lib().sq_budget_stream(ordinal, sm_budget, ctypes.byref(stream), ctypes.byref(actual),
                                    ctypes.byref(total))
    if code == N.SQ_ERR_ARGUMENT:
        raise ValueError(f"writeback SM budget must be between 0 and {total.value}")
    if code != N.SQ_OK:
        raise RuntimeError(f"SM-budget stream unavailable ({N.lib().sq_error_string(code).decode()}); "
                           "use an SM budget of 0 for an unrestricted stream")
    return torch.cuda.ExternalStream(stream.value, device=ordinal), actual.value, total.value


def writeback_resources(device, sm_budget=32):
    """The writeback stream of ``device`` with ``sm_budget`` SMs (0: the whole device)."""
    ordinal = _ordinal(device)
    key = (ordinal, sm_budget)
    cached = _cache.get(key)
    if cached is not None:
        return cached
    total = torch.cuda.get_device_properties(ordinal).multi_processor_count
    if not 0 <= sm_budget <= total:
        raise ValueError(f"writeback SM budget must be between 0 and {total}")
    if sm_budget:
        stream, actual, total = _budget_stream(ordinal, sm_budget)
    else:
        stream, actual = torch.cuda.Stream(device=ordinal), total
    _cache[key] = WritebackResources(stream, sm_budget, actual, total)
    return _cache[key]
