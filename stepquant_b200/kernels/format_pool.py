"""Baseline state formats (stepquant/kernels/format_pool.py, floating.py:20-53).

``Fp32StatePool``: the FP32 baseline on the device kernel ``sq_fp32_step``,
the state stored uncompressed as fp32 [slots, H, K, V].  ``FormatStatePool``:
the symmetric groupwise (sym_int4/6/8_g128) and dual-axis (dsq_int4/6)
formats on the generic tile kernel (``sq_plan.storage`` 2 and 3).  Both keep
PackedStatePool's slot interface (step / encode / decode / wait / clear / copy).
"""
import ctypes

import torch

from .. import _native as N
from .pool import PackedStatePool


class Fp32StatePool:
    def __init__(self, plan, slots, value_dim=128, spec=None, writeback_stream=None):
        if plan.bits.device.type != "cuda":
            raise ValueError("state pool requires CUDA")
        if spec is not None and spec.kind != "fp32":
            raise NotImplementedError(f"Fp32StatePool holds fp32 states; {spec.name} pages are FormatStatePool's")
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
    """Page layout of a baseline-format pool (kernels/format_pool.py:9-27):
    (offsets, rows, columns, page_bytes).  Each key row's codes are one
    little-endian bitstream of ``values * bits / 8`` bytes; then per row the
    symmetric groups' (fp16 scale, fp16 zero point) pairs or the DSQ fp16 row
    scale; then per head the DSQ (fp16 column scale, fp16 zero) pairs."""
    offsets, rows, columns = [], [], []
    cursor = 0
    bits = plan.bits.detach().cpu().flatten().tolist()
    for b in bits:
        if b == 16:
            cursor = (cursor + 1) // 2 * 2
        offsets.append(cursor)
        cursor += values * b // 8
    cursor = (cursor + 3) // 4 * 4
    floating, dual = spec.kind == "fp32", spec.kind == "dsq"
    for b in bits:
        rows.append(cursor if b != 16 and not floating else -1)
        cursor += 0 if floating or b == 16 else (2 if dual else values // spec.group_size * 4)
    cursor = (cursor + 3) // 4 * 4
    for _ in range(plan.bits.shape[0]):
        columns.append(cursor)
        cursor += values * 4 if dual else 0
    return offsets, rows, columns, cursor


class FormatStatePool(PackedStatePool):
    """Baseline-format pages (sym_int*_g128, dsq_int*; kernels/format_pool.py:30-128)
    with the PackedStatePool slot interface, on the generic tile kernel.

    Synchronous only, like the reference's fused format kernels.  The fp32
    format returns an ``Fp32StatePool``.  Codes and scales are exactly the
    reference's ``formats.group_fit`` / ``dual_fit`` of the state.
    """

    def __new__(cls, plan, slots, value_dim, spec, writeback_stream=None, layout=None):
        if spec.kind == "fp32":
            return Fp32StatePool(plan, slots, value_dim, spec, writeback_stream)
        return super().__new__(cls)

    def __init__(self, plan, slots, value_dim, spec, writeback_stream=None, layout=None):
        from ..quantization import DevicePlan
        if writeback_stream is not None:
            raise ValueError("these fused formats require synchronous writeback")
        if spec.kind not in ("symmetric", "dsq"):
            raise ValueError(f"not a baseline state format: {spec.name}")
        if not (plan.bits == spec.bits).all():
            raise ValueError(f"precision map incompatible with {spec.name}")
        if plan.bits.device.type != "cuda":
            raise ValueError("fused format pool requires CUDA")
        self.plan, self.spec = plan, spec
        self.heads, self.keys = plan.bits.shape
        self.values, self.device = value_dim, plan.bits.device
        if self.keys & (self.keys - 1) or value_dim & (value_dim - 1) or value_dim % 4:
            raise ValueError("key/value dimensions must be powers of two, value >= 4")
        if spec.kind == "dsq" and self.keys > 128:
            raise ValueError("dual-axis g128 requires key_dim <=128")
        if spec.kind == "symmetric" and value_dim % spec.group_size:
            raise ValueError("group size must divide value dimension")
        if not 4 <= self.keys <= 128 or value_dim > 128:
            raise NotImplementedError("this build supports key and value dimensions from 4 to 128")
        offsets, rows, columns, page_bytes = format_layout(plan, value_dim, spec) if layout is None else layout
        # The device plan's offset table ends with one (unused) stride per head.
        self._dp = DevicePlan(plan, value_dim, spec.kind, (list(offsets) + [0] * self.heads, rows, columns, page_bytes),
                              group=spec.group_size if spec.kind == "symmetric" else value_dim)
        self.page_bytes = page_bytes
        self.offsets, self.rows, self.columns = self._dp.offsets, self._dp.rows, self._dp.columns
        self.bits, self.impact = self._dp.bits, self._dp.impact
        self.storage = spec.kind
        self.early_writeback = False
        self._storage = torch.zeros(slots * page_bytes + 64, device=self.device, dtype=torch.uint8)
        self.data = self._storage[:slots * page_bytes].view(slots, page_bytes)
        self.status = torch.zeros(1, device=self.device, dtype=torch.int32)
        self.coefficients = None
        self.row_tile = 0
        self._init_writeback(None, 0)
        self._init_workspace(slots, None)
