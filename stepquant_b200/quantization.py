"""Quantization plan, packed codec and fit_state (the reference's ``stepquant.quantization``).

``QuantizationPlan`` keeps the reference's validation (quantization.py:7-30).
``fit_state`` and ``StateCodec`` run on the device through the C ABI
(``sq_fit_state``, ``sq_pack``, ``sq_unpack``); they accept CUDA tensors only.
"""
from dataclasses import dataclass

import torch

from . import _native as N
from .packing import pack, unpack


REFERENCE_WIDTHS = (2, 4, 6, 8)
EXTENDED_WIDTHS = (2, 3, 4, 5, 6, 8)


@dataclass
class QuantizationPlan:
    """A layer's per-row code widths (16: fp16 pivot) and impact factors.

    ``extended_widths=True`` also admits 3- and 5-bit rows, an extension of
    this package (the reference accepts 2, 4, 6, 8 and 16 only).  fit_state
    treats them with the reference's width-generic formula (qmax 2^(b-1) - 1,
    KDA norm 2^(8-b)); codes pack like every other width, and a page row's
    value-tile chunk takes ceil(tile b / 8) bytes (KDA: 2 bytes at 3 bits, 3
    at 5 bits, the tail bits zero).  Plans without the flag keep the
    reference's validation and page layout exactly.
    """
    architecture: str
    bits: torch.Tensor    # [H, K], 16 denotes fp16 pivots
    impact: torch.Tensor  # [H, K], normalized row weights w
    value_group_size: int = 32
    extended_widths: bool = False

    def __post_init__(self):
        if self.architecture not in ("gdn", "kda"):
            raise ValueError("architecture must be gdn or kda")
        if self.bits.ndim != 2 or self.bits.shape != self.impact.shape:
            raise ValueError("bits and impact must have shape [heads, key_dim]")
        allowed = (*EXTENDED_WIDTHS, 16) if self.extended_widths else (*REFERENCE_WIDTHS, 16)
        if not torch.isin(self.bits, torch.tensor(allowed, device=self.bits.device)).all():
            raise ValueError("precision must be 2, 4, 6, 8 or 16")
        if self.architecture == "gdn" and not (self.bits == self.bits[:, :1]).all():
            raise ValueError("GDN allocation is per whole head")
        if not torch.isfinite(self.impact).all() or (self.impact <= 0).any():
            raise ValueError("impact factors must be finite and positive")
        if self.value_group_size < 1:
            raise ValueError("value_group_size must be positive")

    def to(self, device):
        return QuantizationPlan(self.architecture, self.bits.to(device), self.impact.to(device),
                                self.value_group_size, self.extended_widths)

    @property
    def widths(self):
        """The integer code widths this plan may hold."""
        return EXTENDED_WIDTHS if self.extended_widths else REFERENCE_WIDTHS


@dataclass
class PackedState:
    codes: dict
    rows: torch.Tensor
    columns: torch.Tensor
    pivots: torch.Tensor
    two_bit_rows: torch.Tensor | None
    shape: tuple

    @property
    def nbytes(self):
        values = [*self.codes.values(), self.rows, self.columns, self.pivots, self.two_bit_rows]
        return sum(x.numel() * x.element_size() for x in values if x is not None)


class DevicePlan:
    """Device tables of a plan plus its page layout, packed into an ``sq_plan``."""

    # sq_plan.storage codes: STEPQuant packed pages, byte carriers, and the
    # baseline formats (kernels/format_pool.py) symmetric groups and DSQ.
    STORAGE = {"packed": 0, "byte": 1, "symmetric": 2, "dsq": 3}

    def __init__(self, plan, values, storage="packed", layout=None, group=None):
        from .kernels.pool import packed_layout
        N.require_cuda(plan.bits)
        self.plan = plan
        self.device = plan.bits.device
        self.heads, self.keys = plan.bits.shape
        self.values = values
        offsets, rows, columns, page_bytes = layout if layout is not None else packed_layout(plan, values, storage)
        self.page_bytes = page_bytes
        dev = self.device
        self.bits = plan.bits.to(device=dev, dtype=torch.int32).contiguous()
        self.impact = plan.impact.to(device=dev, dtype=torch.float32).contiguous()
        self.offsets = torch.tensor(offsets, device=dev, dtype=torch.int32)
        self.rows = torch.tensor(rows, device=dev, dtype=torch.int32)
        self.columns = torch.tensor(columns, device=dev, dtype=torch.int32)
        self.bits_host = plan.bits.detach().to("cpu", torch.int32).contiguous()
        self.struct = N.SqPlan(
            N.SQ_KDA if plan.architecture == "kda" else N.SQ_GDN, self.heads, self.keys, values,
            plan.value_group_size if group is None else group, self.STORAGE[storage], page_bytes,
            self.bits.data_ptr(), self.impact.data_ptr(),
            self.offsets.data_ptr(), self.rows.data_ptr(), self.columns.data_ptr(), self.bits_host.data_ptr())

    def ref(self):
        import ctypes
        return ctypes.byref(self.struct)


_plans = {}


def _device_plan(plan, values):
    key = (id(plan), plan.bits.data_ptr(), plan.impact.data_ptr(), values)
    entry = _plans.get(key)
    if entry is None or entry.plan is not plan:
        entry = DevicePlan(plan, values)
        _plans[key] = entry
    return entry


def fit_state(x, plan):
    """Integer levels, stored row/column factors and reconstruction (quantization.py:54-98).

    Returns (z int16 [B,H,K,V], r fp16 [B,H,K], c fp16 [B,H,V],
    r2 fp16 [B,H2,K,V/G] for GDN 2-bit heads or None, recon fp32 [B,H,K,V]).
    """
    N.require_cuda(x, plan.bits)
    x = x.float().contiguous()
    batch, heads, keys, values = x.shape
    if (heads, keys) != tuple(plan.bits.shape):
        raise ValueError("state/precision-map shape mismatch")
    dp = _device_plan(plan, values)
    two = int((plan.bits[:, 0] == 2).sum()) if plan.architecture == "gdn" else 0
    if two and values % plan.value_group_size:
        raise ValueError("Qwen INT2 value dimension must be divisible by value_group_size")
    z = torch.empty(x.shape, device=x.device, dtype=torch.int16)
    r = torch.empty((batch, heads, keys), device=x.device, dtype=torch.float16)
    c = torch.empty((batch, heads, values), device=x.device, dtype=torch.float16)
    r2 = torch.empty((batch, two, keys, values // plan.value_group_size), device=x.device,
                     dtype=torch.float16) if two else None
    recon = torch.empty_like(x)
    N.check(N.lib().sq_fit_state(dp.ref(), N.ptr(x), batch, N.ptr(z), N.ptr(r), N.ptr(c), N.ptr(r2),
                                 N.ptr(recon), N.stream_handle()))
    return z, r, c, r2, recon


class StateCodec:
    """Packed persistent storage of a whole state (quantization.py:101-152)."""

    def __init__(self, plan):
        self.plan = plan
        flat = plan.bits.flatten()
        self.widths = getattr(plan, "widths", REFERENCE_WIDTHS)
        self.indices = {b: (flat == b).nonzero().flatten() for b in (*self.widths, 16)}
        self.integer_rows = (flat != 16).nonzero().flatten()
        self.integer_heads = (plan.bits != 16).any(-1).nonzero().flatten()
        self.two_heads = (plan.bits[:, 0] == 2).nonzero().flatten() if plan.architecture == "gdn" else None

    def encode(self, state):
        if tuple(state.shape[1:3]) != tuple(self.plan.bits.shape):
            raise ValueError("state/precision-map shape mismatch")
        z, r, c, r2, _ = fit_state(state, self.plan)
        batch, heads, keys, values = state.shape
        z = z.reshape(batch, heads * keys, values)
        packed = {}
        for bits in self.widths:
            codes = z[:, self.indices[bits]]
            if bits == 2 and self.plan.architecture == "gdn":
                codes = torch.div(codes + 3, 2, rounding_mode="floor")
            else:
                codes = codes + (2 ** (bits - 1) - 1)
            packed[bits] = pack(codes.to(torch.int16), bits, extended=True)
        pivots = state.reshape(batch, heads * keys, values)[:, self.indices[16]].half()
        return PackedState(packed, r.reshape(batch, -1)[:, self.integer_rows], c[:, self.integer_heads],
                           pivots, r2, tuple(state.shape))

    def decode(self, packed):
        batch, heads, keys, values = packed.shape
        device = packed.rows.device
        N.require_cuda(packed.rows)
        z = torch.zeros((batch, heads * keys, values), device=device)
        for bits in self.widths:
            idx = self.indices[bits]
            codes = unpack(packed.codes[bits], bits, batch * idx.numel() * values,
                           extended=True).reshape(batch, -1, values).float()
            if bits == 2 and self.plan.architecture == "gdn":
                codes = 2 * codes - 3
            else:
                codes -= 2 ** (bits - 1) - 1
            if self.plan.architecture == "kda":
                codes *= 2 ** (8 - bits)
            z[:, idx] = codes
        r = torch.ones((batch, heads * keys), device=device)
        r[:, self.integer_rows] = packed.rows.float()
        c = torch.ones((batch, heads, values), device=device)
        c[:, self.integer_heads] = packed.columns.float()
        result = z.reshape(batch, heads, keys, values) * r.reshape(batch, heads, keys, 1) * c.unsqueeze(-2)
        if packed.two_bit_rows is not None:
            result[:, self.two_heads] = (z.reshape(batch, heads, keys, values)[:, self.two_heads]
                                         * packed.two_bit_rows.float().repeat_interleave(self.plan.value_group_size, -1)
                                         * c[:, self.two_heads, None, :])
        result.reshape(batch, heads * keys, values)[:, self.indices[16]] = packed.pivots.float()
        return result
