"""stepquant_b200: B200-native (sm_100a) packed-state recurrent decode path of STEPQuant.

Host code in Python mirrors the reference API (``formats``, ``packing``,
``quantization``, ``kernels.pool``, ``kernels.writeback``, ``sglang``); the
arithmetic runs in libstepquant_b200.so through the C ABI declared in
include/stepquant_b200.h.  State coordinates are [batch, head, key, value].
"""
from .quantization import PackedState, QuantizationPlan, StateCodec, fit_state

__all__ = ["PackedState", "QuantizationPlan", "StateCodec", "fit_state"]
