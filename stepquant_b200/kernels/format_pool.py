"""FP32 state pool: the reference's FP32 baseline format (stepquant/kernels/format_pool.py,
floating.py:20-53) on the device kernel ``sq_fp32_step``.

Same slot interface as PackedStatePool (step / encode / decode / wait / clear /
copy); the state is stored uncompressed as fp32 [slots, H, K, V].  The other
baseline formats (sym_int*, dsq_*) are not built.
"""
import ctypes

import torch

from .. import _native as N


class Fp32StatePool:
    def __init__(self, plan, slots, value_dim=128, spec=None, writeback_stream=None):
        if plan.bits.device.type != "cuda":
            raise ValueError("state pool requires CUDA")
        if spec is not None and spec.kind != "fp32":
            raise NotImplementedError(f"state format {spec.name} has no device pool in this build (fp32 only)")
        self.plan = plan
        self.heads, self.keys = plan.bits.shape
        self.values = value_dim
        self.device = plan.bits.device
        self.data = torch.zeros(slots, self.heads, self.keys, value_dim, device=self.device)
        self.status = torch.zeros(1, device=self.device, dtype=torch.int32)
        self.writeback_stream = None
        self.pending = False
        self.deferred = None

    @property
    def nbytes(self):
        return self.data.numel() * 4

    def wait(self):
        pass

    def encode(self, state, slots):
        if state.shape != (slots.numel(), self.heads, self.keys, self.values):
            raise ValueError("state must be [active slots, heads, key, value]")
        active = slots > 0
        self.data[slots[active]] = state[active].float()

    def decode(self, slots):
        out = torch.zeros(slots.numel(), self.heads, self.keys, self.values, device=self.device)
        active = slots > 0
        out[active] = self.data[slots[active]]
        return out

    def step(self, q, k, v, g, beta, slots, *, normalize=False, scale=1., a_log=None, dt_bias=None):
        batch = slots.numel()
        if not batch:
            return torch.empty((0, self.heads, self.values), device=q.device, dtype=q.dtype)
        q = q.reshape(batch, -1, self.keys)
        k = k.reshape(batch, -1, self.keys).to(q.dtype)
        v = v.reshape(batch, self.heads, self.values).to(q.dtype)
        if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
            raise ValueError("head coordinates must be contiguous")
        g, beta = g.contiguous(), beta.contiguous().to(g.dtype)
        slots = slots.to(device=self.device, dtype=torch.int64).contiguous()
        out = torch.empty((batch, self.heads, self.values), device=q.device, dtype=q.dtype)
        if a_log is not None:
            a_log, dt_bias = a_log.float().contiguous(), dt_bias.float().contiguous()
        args = N.SqStepArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), k.stride(0), v.stride(0), q.shape[1],
                            N.dtype_code(q.dtype), g.data_ptr(), beta.data_ptr(), N.dtype_code(g.dtype),
                            int(bool(normalize)), None if a_log is None else a_log.data_ptr(),
                            None if dt_bias is None else dt_bias.data_ptr(), float(scale), 0, out.data_ptr())
        N.check(N.lib().sq_fp32_step(N.ptr(self.data), self.data.shape[0], self.heads, self.keys, self.values,
                                     int(self.plan.architecture == "kda"), N.ptr(slots), batch, ctypes.byref(args),
                                     N.ptr(self.status), N.stream_handle()))
        return out

    def clear(self, slots):
        self.data[slots] = 0

    def copy(self, source, destination):
        self.data[destination] = self.data[source]


def format_layout(plan, values, spec):
    """Bytes per slot of a baseline-format page (fp32 only in this build)."""
    if spec.kind != "fp32":
        raise NotImplementedError(f"state format {spec.name} is not built")
    heads, keys = plan.bits.shape
    return None, None, None, heads * keys * values * 4
