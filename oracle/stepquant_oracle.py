"""CPU oracle for the packed-state decode path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker (or as the timed CPU port).  The
product path (``stepquant_b200``) never imports it and has no CPU fallback.

This is a numpy restatement of the reference STEPQuant torch path:

* ``fit_state``       -> stepquant/quantization.py:54-98
* ``codec_encode``    -> stepquant/quantization.py:109-126  (StateCodec.encode)
* ``codec_decode``    -> stepquant/quantization.py:128-152  (StateCodec.decode)
* ``pack/unpack``     -> stepquant/packing.py:6-22
* ``packed_layout``   -> stepquant/kernels/pool.py:19-66
* ``page_encode``     -> pool page image written by pool.encode
                         (kernels/pool.py:184-190,319-331; fused.py:252-282 rows,
                         fused.py:63-127 columns/codes; bitpack.py:7-30 word order)
* ``page_decode``     -> fused.py:19-59 (codec_kernel / _read)
* ``delta_step``      -> stepquant/core.py:5-15
* ``prepare_inputs``  -> fused.py:156-179 and readout.py:22-39 (q/k L2 norm,
                         scale, GQA head map, raw gate transform)
* ``decode_step``     -> PackedStatePool.step + writeback (kernels/pool.py:200-316)
                         with the sync semantics of core.delta_step + fit_state.

Bit-exactness.  ``fit_state`` in the reference sums in fp32 with torch's CPU
reductions.  Their order is part of the result (a different order moves an fp32
sum by an ulp, which occasionally moves an fp16 scale by one step).  The two
sums it takes are restated here in torch 2.11's CPU order:

* ``torch_inner_sum``: ``x.abs().mean(-1)`` over a contiguous row (aten
  SumKernel ``cascade_sum`` -> ``vectorized_inner_sum`` with 8-lane fp32
  vectors, a 4-way interleaved ``row_sum`` and an in-order lane sum).
* ``torch_outer_sum``: ``(...).sum(-2)`` over the key axis (``vectorized_outer_sum``
  / ``scalar_outer_sum`` with the 16-row ``multi_row_sum`` cascade).

The restatement is pinned against the reference itself: ``tests/golden`` holds
vectors produced by the unmodified reference (``tests/golden/make_golden.py``)
and ``tests/test_oracle_golden.py`` requires byte equality.  Every other step
is elementwise IEEE fp32 arithmetic in the reference's operation order.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

F32 = np.float32
_LANES = 8  # fp32 lanes of the Vectorized<float> the torch CPU sum kernel uses


# ---------------------------------------------------------------------------
# torch CPU summation orders
# ---------------------------------------------------------------------------

def _add(a, b):
    return (a + b).astype(F32, copy=False)


def _cascade(rows, nrows):
    """aten ``multi_row_sum``: ``rows[i][k]`` summed over i for each k.

    Sixteen consecutive rows accumulate in order into level 0; finished blocks
    are carried into higher levels, which are added back at the end.
    """
    size = len(rows)
    ceil_log2 = 0 if size <= 1 else math.ceil(math.log2(size))
    level_power = max(4, ceil_log2 // 4)
    level_step = 1 << level_power
    level_mask = level_step - 1
    shape = np.shape(rows[0][0]) if size else ()
    acc = [[np.zeros(shape, F32) for _ in range(nrows)] for _ in range(4)]
    i = 0
    while i + level_step <= size:
        for _ in range(level_step):
            for k in range(nrows):
                acc[0][k] = _add(acc[0][k], rows[i][k])
            i += 1
        for j in range(1, 4):
            for k in range(nrows):
                acc[j][k] = _add(acc[j][k], acc[j - 1][k])
                acc[j - 1][k] = np.zeros(shape, F32)
            if i & (level_mask << (j * level_power)):
                break
    while i < size:
        for k in range(nrows):
            acc[0][k] = _add(acc[0][k], rows[i][k])
        i += 1
    for j in range(1, 4):
        for k in range(nrows):
            acc[0][k] = _add(acc[0][k], acc[j][k])
    return acc[0]


def _row_sum(items, template):
    """aten ``row_sum``: a 4-way interleaved cascade, then the 4 partials in order."""
    size = len(items)
    size_ilp = size // 4
    if size_ilp:
        acc = _cascade([[items[4 * i + k] for k in range(4)] for i in range(size_ilp)], 4)
    else:
        acc = [np.zeros_like(template) for _ in range(4)]
    for i in range(size_ilp * 4, size):
        acc[0] = _add(acc[0], items[i])
    total = acc[0]
    for k in range(1, 4):
        total = _add(total, acc[k])
    return total


def torch_inner_sum(x):
    """Sum over the last (contiguous) axis in torch 2.11's CPU fp32 order."""
    x = np.asarray(x, F32)
    n = x.shape[-1]
    if n >= _LANES:
        nv = n // _LANES
        vectors = [x[..., _LANES * m:_LANES * (m + 1)] for m in range(nv)]
        lanes = _row_sum(vectors, vectors[0])
        total = np.zeros(x.shape[:-1], F32)
        for i in range(nv * _LANES, n):
            total = _add(total, x[..., i])
        for lane in range(_LANES):
            total = _add(total, lanes[..., lane])
        return total
    return _row_sum([x[..., i] for i in range(n)], x[..., 0])


def torch_outer_sum(x):
    """Sum over axis -2 of a contiguous ``[..., K, V]`` array in torch's CPU order."""
    x = np.asarray(x, F32)
    keys, values = x.shape[-2], x.shape[-1]
    rows = [x[..., k, :] for k in range(keys)]
    out = np.empty(x.shape[:-2] + (values,), F32)
    j = 0
    if values >= _LANES:
        while j + 4 * _LANES <= values:
            res = _cascade([[rows[i][..., j + _LANES * m:j + _LANES * (m + 1)] for m in range(4)]
                            for i in range(keys)], 4)
            for m in range(4):
                out[..., j + _LANES * m:j + _LANES * (m + 1)] = res[m]
            j += 4 * _LANES
        while j + _LANES <= values:
            out[..., j:j + _LANES] = _row_sum([rows[i][..., j:j + _LANES] for i in range(keys)],
                                               rows[0][..., j:j + _LANES])
            j += _LANES
        for jj in range(j, values):  # not reached for power-of-two value dims
            out[..., jj] = _row_sum([rows[i][..., jj] for i in range(keys)], rows[0][..., jj])
        return out
    while j + 3 < values:
        res = _cascade([[rows[i][..., j + m] for m in range(4)] for i in range(keys)], 4)
        for m in range(4):
            out[..., j + m] = res[m]
        j += 4
    for jj in range(j, values):
        out[..., jj] = _row_sum([rows[i][..., jj] for i in range(keys)], rows[0][..., jj])
    return out


# ---------------------------------------------------------------------------
# plan and quantizer
# ---------------------------------------------------------------------------

@dataclass
class Plan:
    """Mirror of QuantizationPlan (quantization.py:7-26) as numpy arrays.

    ``extended_widths`` admits 3- and 5-bit rows: this build's labelled
    extension (the reference rejects them, quantization.py:19-20).  fit_state
    is the reference's formula unchanged at those widths (qmax 2^(b-1) - 1,
    KDA norm 2^(8-b)); codes pack as the reference packs every width (code i
    at bit i b), and a page row's tile chunk takes ceil(tile b / 8) bytes
    (KDA tiles of 4 values: 2 bytes at 3 bits, 3 at 5 bits, tail bits zero).
    """
    architecture: str
    bits: np.ndarray     # [H, K] int, 16 = fp16 pivot
    impact: np.ndarray   # [H, K] float32
    value_group_size: int = 32
    extended_widths: bool = False

    def __post_init__(self):
        self.bits = np.asarray(self.bits).astype(np.int64)
        self.impact = np.asarray(self.impact, F32)
        if self.architecture not in ("gdn", "kda"):
            raise ValueError("architecture must be gdn or kda")
        if self.bits.ndim != 2 or self.bits.shape != self.impact.shape:
            raise ValueError("bits and impact must have shape [heads, key_dim]")
        allowed = [2, 3, 4, 5, 6, 8, 16] if self.extended_widths else [2, 4, 6, 8, 16]
        if not np.isin(self.bits, allowed).all():
            raise ValueError("precision must be 2, 4, 6, 8 or 16")
        if self.architecture == "gdn" and not (self.bits == self.bits[:, :1]).all():
            raise ValueError("GDN allocation is per whole head")
        if not np.isfinite(self.impact).all() or (self.impact <= 0).any():
            raise ValueError("impact factors must be finite and positive")


def fp16_scale(x):
    """quantization.py:49-51: clamp to the fp16 range, round to fp16 (RNE)."""
    return np.clip(np.asarray(x, F32), F32(2.0 ** -24), F32(65504)).astype(np.float16).astype(F32)


def fit_state(x, plan: Plan):
    """quantization.py:54-98; returns z int16, r fp16, c fp16, r2 fp16|None, recon f32."""
    x = np.asarray(x, F32)
    bits = plan.bits
    w = plan.impact[None, :, :, None]
    integer = (bits != 16)[None, :, :, None]
    clamped = np.minimum(bits, 8).astype(F32)
    qmax = (np.ldexp(F32(1), (clamped - 1).astype(np.int32)) - 1).astype(F32)[None, :, :, None]
    if plan.architecture == "kda":
        norm = np.ldexp(F32(1), (8 - clamped).astype(np.int32)).astype(F32)[None, :, :, None]
    else:
        norm = np.ones_like(qmax)
    mean = torch_inner_sum(np.abs(x))[..., None] / F32(x.shape[-1])
    r = fp16_scale(np.sqrt((np.maximum(mean, F32(1e-20)) / w).astype(F32)))
    r_full = np.broadcast_to(r, x.shape).copy()
    qmax = np.broadcast_to(qmax, (1,) + bits.shape + (1,)).copy()
    two_rows = None
    if plan.architecture == "gdn":
        two_heads = bits[:, 0] == 2
    else:
        two_heads = np.zeros(bits.shape[0], bool)
    if two_heads.any():
        group = plan.value_group_size
        if x.shape[-1] % group:
            raise ValueError("Qwen INT2 value dimension must be divisible by value_group_size")
        sub = x[:, two_heads]
        grouped = np.abs(sub).reshape(*sub.shape[:-1], -1, group)
        gmean = torch_inner_sum(grouped) / F32(group)
        two_rows = fp16_scale(np.sqrt((np.maximum(gmean, F32(1e-20)) / w[:, two_heads]).astype(F32)))
        r_full[:, two_heads] = np.repeat(two_rows, group, axis=-1)
        qmax[:, two_heads] = F32(3)
    scaled = (x / r_full).astype(F32)
    limit = (qmax * norm).astype(F32)
    c = fp16_scale(np.where(integer, (np.abs(scaled) / limit).astype(F32), F32(0)).max(-2, keepdims=True))

    def encode(columns):
        y = ((scaled / columns).astype(F32) / norm).astype(F32)
        z = np.minimum(np.maximum(np.rint(y), -qmax), qmax).astype(F32)
        if two_heads.any():
            y2 = y[:, two_heads]
            z[:, two_heads] = np.where(y2 >= 0, F32(1), F32(-1)) * np.where(np.abs(y2) >= 2, F32(3), F32(1))
        return z

    z = encode(c)
    v = ((r_full * norm).astype(F32) * z).astype(F32)
    weights = ((w * w).astype(F32) * integer).astype(F32)
    num = torch_outer_sum(((weights * v).astype(F32) * x).astype(F32))[..., None, :]
    den = torch_outer_sum((weights * (v * v).astype(F32)).astype(F32))[..., None, :]
    ratio = (num / np.maximum(den, F32(1e-30))).astype(F32)
    c = fp16_scale(np.where(den > 0, ratio, c))
    z = encode(c)
    recon = ((r_full * c).astype(F32) * norm).astype(F32)
    recon = (recon * z).astype(F32)
    recon = np.where(integer, recon, x.astype(np.float16).astype(F32))
    return (z.astype(np.int16), r[..., 0].astype(np.float16), c[:, :, 0, :].astype(np.float16),
            None if two_rows is None else two_rows.astype(np.float16), recon.astype(F32))


# ---------------------------------------------------------------------------
# packing and the StateCodec byte streams
# ---------------------------------------------------------------------------

def widths(plan):
    """The integer code widths a plan may hold."""
    return (2, 3, 4, 5, 6, 8) if getattr(plan, "extended_widths", False) else (2, 4, 6, 8)


def chunk_bytes(tile, bits):
    """Bytes of one row's value-tile chunk (tile * bits / 8 at the reference's widths)."""
    return (tile * bits + 7) // 8


def pack(codes, bits, extended=False):
    """packing.py:6-14: little-endian, n = 8/gcd(b,8) codes per n*b/8 bytes
    (``extended``: also 3 and 5 bits, 8 codes per 3 or 5 bytes)."""
    if bits not in ((2, 3, 4, 5, 6, 8) if extended else (2, 4, 6, 8)):
        raise ValueError("supported code widths: 2, 4, 6, 8")
    flat = np.asarray(codes).reshape(-1).astype(np.int64)
    n = 8 // math.gcd(bits, 8)
    width = n * bits // 8
    flat = np.pad(flat, (0, (-flat.size) % n)).reshape(-1, n)
    word = (flat << (np.arange(n) * bits)).sum(-1)
    return ((word[:, None] >> (np.arange(width) * 8)) & 255).astype(np.uint8).reshape(-1)


def unpack(data, bits, count):
    """packing.py:17-22."""
    n = 8 // math.gcd(bits, 8)
    width = n * bits // 8
    word = (np.asarray(data).astype(np.int64).reshape(-1, width) << (np.arange(width) * 8)).sum(-1)
    codes = (word[:, None] >> (np.arange(n) * bits)) & ((1 << bits) - 1)
    return codes.reshape(-1)[:count].astype(np.int16)


def codec_encode(state, plan: Plan):
    """StateCodec.encode (quantization.py:109-126) -> dict of numpy byte streams."""
    state = np.asarray(state, F32)
    if tuple(state.shape[1:3]) != tuple(plan.bits.shape):
        raise ValueError("state/precision-map shape mismatch")
    z, r, c, r2, _ = fit_state(state, plan)
    batch, heads, keys, values = state.shape
    flat_bits = plan.bits.reshape(-1)
    z = z.reshape(batch, heads * keys, values).astype(np.int64)
    codes = {}
    for b in widths(plan):
        idx = np.nonzero(flat_bits == b)[0]
        sel = z[:, idx]
        if b == 2 and plan.architecture == "gdn":
            sel = (sel + 3) // 2
        else:
            sel = sel + (2 ** (b - 1) - 1)
        codes[b] = pack(sel, b, extended=True)
    integer_rows = np.nonzero(flat_bits != 16)[0]
    integer_heads = np.nonzero((plan.bits != 16).any(-1))[0]
    pivots = state.reshape(batch, heads * keys, values)[:, np.nonzero(flat_bits == 16)[0]].astype(np.float16)
    return dict(codes=codes, rows=r.reshape(batch, -1)[:, integer_rows], columns=c[:, integer_heads],
                pivots=pivots, two_bit_rows=r2, shape=state.shape)


def codec_decode(packed, plan: Plan):
    """StateCodec.decode (quantization.py:128-152)."""
    batch, heads, keys, values = packed["shape"]
    flat_bits = plan.bits.reshape(-1)
    z = np.zeros((batch, heads * keys, values), F32)
    for b in widths(plan):
        idx = np.nonzero(flat_bits == b)[0]
        codes = unpack(packed["codes"][b], b, batch * idx.size * values).reshape(batch, -1, values).astype(F32)
        if b == 2 and plan.architecture == "gdn":
            codes = 2 * codes - 3
        else:
            codes = codes - (2 ** (b - 1) - 1)
        if plan.architecture == "kda":
            codes = codes * F32(2 ** (8 - b))
        z[:, idx] = codes
    r = np.ones((batch, heads * keys), F32)
    r[:, flat_bits != 16] = packed["rows"].astype(F32)
    c = np.ones((batch, heads, values), F32)
    c[:, (plan.bits != 16).any(-1)] = packed["columns"].astype(F32)
    z4 = z.reshape(batch, heads, keys, values)
    result = ((z4 * r.reshape(batch, heads, keys, 1)).astype(F32) * c[:, :, None, :]).astype(F32)
    if packed["two_bit_rows"] is not None:
        two_heads = np.nonzero(plan.bits[:, 0] == 2)[0]
        rep = np.repeat(packed["two_bit_rows"].astype(F32), plan.value_group_size, axis=-1)
        result[:, two_heads] = ((z4[:, two_heads] * rep).astype(F32) * c[:, two_heads, None, :]).astype(F32)
    result = result.reshape(batch, heads * keys, values)
    result[:, flat_bits == 16] = packed["pivots"].astype(F32)
    return result.reshape(batch, heads, keys, values)


# ---------------------------------------------------------------------------
# pool page layout and page images
# ---------------------------------------------------------------------------

def packed_layout(plan: Plan, value_dim, storage="packed"):
    """kernels/pool.py:19-66: (offsets, rows, columns, page_bytes)."""
    if storage not in ("packed", "byte"):
        raise ValueError("state storage must be packed or byte")
    bits = plan.bits.tolist()
    offsets, rows, columns = [], [], []
    cursor = 0
    tile = min(4 if plan.architecture == "kda" else 16, value_dim)
    strides = []
    if storage == "byte":
        for head in bits:
            code_base = cursor
            if any(b != 16 for b in head):
                cursor += len(head) * value_dim
            pivot_base = cursor
            pivot_index = 0
            for i, b in enumerate(head):
                if b == 16:
                    offsets.append(pivot_base + 2 * pivot_index * value_dim)
                    pivot_index += 1
                else:
                    offsets.append(code_base + i)
            cursor += 2 * sum(b == 16 for b in head) * value_dim
            strides.append(code_base)
    else:
        for head in bits:
            local = 0
            for b in head:
                if b == 16:
                    local = (local + 1) // 2 * 2
                offsets.append(cursor + local)
                local += chunk_bytes(tile, b)
            stride = (local + 1) // 2 * 2
            strides.append(stride)
            cursor += stride * (value_dim // tile)
    offsets.extend(strides)
    cursor = (cursor + 1) // 2 * 2
    for head in bits:
        for b in head:
            rows.append(cursor if b != 16 else -1)
            if b != 16:
                cursor += 2 * (value_dim // plan.value_group_size if b == 2 and plan.architecture == "gdn" else 1)
    for head in bits:
        columns.append(cursor if any(b != 16 for b in head) else -1)
        if any(b != 16 for b in head):
            cursor += 2 * value_dim
    if storage == "byte":
        cursor = (cursor + 15) // 16 * 16
    return offsets, rows, columns, cursor


def _put_half(page, byte_offset, value):
    page[byte_offset:byte_offset + 2] = np.frombuffer(np.float16(value).tobytes(), np.uint8)


def _get_half(page, byte_offset):
    return np.frombuffer(page[byte_offset:byte_offset + 2].tobytes(), np.float16)[0]


def _tile(plan, values):
    return min(4 if plan.architecture == "kda" else 16, values)


def page_store(page, plan: Plan, values, z, r, c, r2, pivots_f16):
    """Write one request's fitted state into its (packed) page image in place.

    Only the bytes the reference kernels store are written: code bits of
    integer rows (bitpack.py:7-30, fit.py:114-148), fp16 pivots
    (fused.py:272-273), r / GDN 2-bit group r (fused.py:274-282) and c
    (fused.py:127).  Alignment padding keeps its previous contents.
    """
    heads, keys = plan.bits.shape
    offsets, rows, columns, _ = packed_layout(plan, values)
    tile = _tile(plan, values)
    strides = offsets[heads * keys:]
    two_index = 0
    for h in range(heads):
        stride = strides[h]
        b0 = int(plan.bits[h, 0])
        if (plan.bits[h] == b0).all() and b0 in (4, 6, 8) and stride == keys * tile * b0 // 8:
            # Uniform head: its code region is one little-endian bitstream in
            # (value tile, key row, lane) order.
            codes = z[h].astype(np.int64) + (2 ** (b0 - 1) - 1)
            stream = codes.reshape(keys, values // tile, tile).transpose(1, 0, 2).reshape(-1)
            region = pack(stream, b0)
            page[offsets[h * keys]:offsets[h * keys] + region.size] = region
            r_bytes = r[h].astype(np.float16).view(np.uint8)
            page[rows[h * keys]:rows[h * keys] + 2 * keys] = r_bytes
            page[columns[h]:columns[h] + 2 * values] = c[h].astype(np.float16).view(np.uint8)
            continue
        for k in range(keys):
            b = int(plan.bits[h, k])
            off = offsets[h * keys + k]
            for t in range(values // tile):
                base = off + t * stride
                if b == 16:
                    for u in range(tile):
                        _put_half(page, base + 2 * u, pivots_f16[h, k, t * tile + u])
                    continue
                if b == 2 and plan.architecture == "gdn":
                    codes = (z[h, k, t * tile:(t + 1) * tile].astype(np.int64) + 3) // 2
                else:
                    codes = z[h, k, t * tile:(t + 1) * tile].astype(np.int64) + (2 ** (b - 1) - 1)
                word = 0
                for u, code in enumerate(codes):
                    word |= int(code) << (u * b)
                nbytes = chunk_bytes(tile, b)
                page[base:base + nbytes] = np.frombuffer(word.to_bytes(nbytes, "little"), np.uint8)
            if b != 16:
                if b == 2 and plan.architecture == "gdn":
                    for g in range(values // plan.value_group_size):
                        _put_half(page, rows[h * keys + k] + 2 * g, r2[two_index, k, g])
                else:
                    _put_half(page, rows[h * keys + k], r[h, k])
        if plan.architecture == "gdn" and plan.bits[h, 0] == 2:
            two_index += 1
        if columns[h] >= 0:
            for v in range(values):
                _put_half(page, columns[h] + 2 * v, c[h, v])


def page_store_byte(page, plan: Plan, values, z, r, c, r2, pivots_f16):
    """Byte-carrier page image of one request (storage='byte'), in place.

    Integer rows keep their signed level as one int8 at code_base + k + v*K
    (KDA: the level times 2^(8-b); fit.py:111-115, kernels/pool.py:29-43);
    fp16 pivot rows are contiguous at their offset; r (GDN 2-bit: per value
    group) and c as in packed pages.
    """
    heads, keys = plan.bits.shape
    offsets, rows, columns, _ = packed_layout(plan, values, "byte")
    kda = plan.architecture == "kda"
    two_index = 0
    for h in range(heads):
        code_base = offsets[heads * keys + h]
        for k in range(keys):
            b = int(plan.bits[h, k])
            off = offsets[h * keys + k]
            if b == 16:
                page[off:off + 2 * values] = pivots_f16[h, k].astype(np.float16).view(np.uint8)
                continue
            level = z[h, k].astype(np.int64) * ((1 << (8 - min(b, 8))) if kda else 1)
            idx = code_base + k + np.arange(values) * keys
            page[idx] = level.astype(np.int8).view(np.uint8)
            if b == 2 and not kda:
                for g in range(values // plan.value_group_size):
                    _put_half(page, rows[h * keys + k] + 2 * g, r2[two_index, k, g])
            else:
                _put_half(page, rows[h * keys + k], r[h, k])
        if not kda and plan.bits[h, 0] == 2:
            two_index += 1
        if columns[h] >= 0:
            page[columns[h]:columns[h] + 2 * values] = c[h].astype(np.float16).view(np.uint8)


def page_encode(state, plan: Plan, pages=None, storage="packed"):
    """pool.encode (kernels/pool.py:184-190,319-331): dense fp32 [B,H,K,V] -> pages [B,P].

    ``pages`` supplies the prior page contents (kept in alignment padding);
    zero pages are used when it is None.  ``storage`` selects packed codes or
    byte carriers.
    """
    state = np.asarray(state, F32)
    batch, heads, keys, values = state.shape
    page_bytes = packed_layout(plan, values, storage)[-1]
    out = np.zeros((batch, page_bytes), np.uint8) if pages is None else np.array(pages, np.uint8)
    if batch == 0:
        return out
    z, r, c, r2, _ = fit_state(state, plan)
    pivots = state.astype(np.float16)
    store = page_store_byte if storage == "byte" else page_store
    for i in range(batch):
        store(out[i], plan, values, z[i], r[i], c[i], None if r2 is None else r2[i], pivots[i])
    return out


def page_decode_byte(pages, plan: Plan, values):
    """byte_codec.py:6-27: byte-carrier pages [B,P] -> dense fp32 [B,H,K,V], x = (r c) z."""
    pages = np.asarray(pages, np.uint8)
    heads, keys = plan.bits.shape
    offsets, rows, columns, _ = packed_layout(plan, values, "byte")
    group = plan.value_group_size
    kda = plan.architecture == "kda"
    out = np.zeros((pages.shape[0], heads, keys, values), F32)
    for i in range(pages.shape[0]):
        page = pages[i]
        for h in range(heads):
            code_base = offsets[heads * keys + h]
            col = np.zeros(values, F32)
            if columns[h] >= 0:
                col = np.frombuffer(page[columns[h]:columns[h] + 2 * values].tobytes(), np.float16).astype(F32)
            for k in range(keys):
                b = int(plan.bits[h, k])
                off = offsets[h * keys + k]
                if b == 16:
                    out[i, h, k] = np.frombuffer(page[off:off + 2 * values].tobytes(), np.float16).astype(F32)
                    continue
                zz = page[code_base + k + np.arange(values) * keys].view(np.int8).astype(F32)
                if b == 2 and not kda:
                    rr = np.array([_get_half(page, rows[h * keys + k] + 2 * (v // group)) for v in range(values)],
                                  np.float16).astype(F32)
                else:
                    rr = np.full(values, _get_half(page, rows[h * keys + k]), np.float16).astype(F32)
                out[i, h, k] = ((rr * col).astype(F32) * zz).astype(F32)
    return out


def page_decode(pages, plan: Plan, values, storage="packed"):
    """fused.py:19-59: pages [B,P] uint8 -> dense fp32 [B,H,K,V]."""
    if storage == "byte":
        return page_decode_byte(pages, plan, values)
    pages = np.asarray(pages, np.uint8)
    heads, keys = plan.bits.shape
    offsets, rows, columns, _ = packed_layout(plan, values)
    tile = _tile(plan, values)
    strides = offsets[heads * keys:]
    out = np.zeros((pages.shape[0], heads, keys, values), F32)
    group = plan.value_group_size
    for i in range(pages.shape[0]):
        page = pages[i]
        for h in range(heads):
            col = np.zeros(values, F32)
            if columns[h] >= 0:
                col = np.frombuffer(page[columns[h]:columns[h] + 2 * values].tobytes(), np.float16).astype(F32)
            b0 = int(plan.bits[h, 0])
            if (plan.bits[h] == b0).all() and b0 in (4, 6, 8) and strides[h] == keys * tile * b0 // 8:
                nbytes = keys * values * b0 // 8
                codes = unpack(page[offsets[h * keys]:offsets[h * keys] + nbytes], b0, keys * values)
                codes = codes.reshape(values // tile, keys, tile).transpose(1, 0, 2).reshape(keys, values)
                zz = (codes.astype(np.int64) - ((1 << (b0 - 1)) - 1)).astype(F32)
                if plan.architecture == "kda":
                    zz = zz * F32(1 << (8 - b0))
                rr = np.frombuffer(page[rows[h * keys]:rows[h * keys] + 2 * keys].tobytes(), np.float16).astype(F32)
                out[i, h] = ((rr[:, None] * col[None, :]).astype(F32) * zz).astype(F32)
                continue
            for k in range(keys):
                b = int(plan.bits[h, k])
                off = offsets[h * keys + k]
                row_vals = np.empty(values, F32)
                for t in range(values // tile):
                    base = off + t * strides[h]
                    if b == 16:
                        row_vals[t * tile:(t + 1) * tile] = np.frombuffer(
                            page[base:base + 2 * tile].tobytes(), np.float16).astype(F32)
                        continue
                    nbytes = chunk_bytes(tile, b)
                    word = int.from_bytes(page[base:base + nbytes].tobytes(), "little")
                    codes = np.array([(word >> (u * b)) & ((1 << b) - 1) for u in range(tile)], np.int64)
                    if b == 2 and plan.architecture == "gdn":
                        zz = (2 * codes - 3).astype(F32)
                    else:
                        zz = (codes - ((1 << (b - 1)) - 1)).astype(F32)
                        if plan.architecture == "kda":
                            zz = zz * F32(1 << (8 - b))
                    if b == 2 and plan.architecture == "gdn":
                        rr = np.array([_get_half(page, rows[h * keys + k] + 2 * ((t * tile + u) // group))
                                       for u in range(tile)], np.float16).astype(F32)
                    else:
                        rr = np.full(tile, _get_half(page, rows[h * keys + k]), np.float16).astype(F32)
                    row_vals[t * tile:(t + 1) * tile] = ((rr * col[t * tile:(t + 1) * tile]).astype(F32) * zz).astype(F32)
                out[i, h, k] = row_vals
    return out


# ---------------------------------------------------------------------------
# recurrent update and input preparation
# ---------------------------------------------------------------------------

def delta_step(state, q, k, v, log_decay, beta):
    """core.py:5-15 in fp32 (the einsums are evaluated in float64 and rounded)."""
    state = np.asarray(state, F32)
    q, k, v, beta = (np.asarray(a, F32) for a in (q, k, v, beta))
    decay = np.exp(np.asarray(log_decay, F32)).astype(F32)
    if decay.ndim == k.ndim - 1:
        decay = decay[..., None]
    retained = (state * decay[..., None]).astype(F32)
    kr = np.einsum("bhk,bhkv->bhv", k.astype(np.float64), retained.astype(np.float64)).astype(F32)
    residual = (v - kr).astype(F32)
    updated = (retained + (k[..., None] * (beta[..., None] * residual)[..., None, :]).astype(F32)).astype(F32)
    output = np.einsum("bhk,bhkv->bhv", q.astype(np.float64), updated.astype(np.float64)).astype(F32)
    return output, updated


def _softplus_gate(u):
    return np.where(u > 20.0, u, np.log1p(np.exp(np.minimum(u, 20.0)))).astype(F32)


def prepare_inputs(q, k, g, beta, heads, *, kda, normalize=False, scale=1.0, a_log=None, dt_bias=None):
    """fused.py:156-179 / readout.py:22-39.

    q, k: [B, HK, K]; g: [B, H] (GDN) or [B, H, K] (KDA) log-decay, or the raw
    gate input when ``a_log`` is given; beta: [B, H] (raw logits when ``a_log``).
    Returns q', k' [B, H, K], log-decay and beta in fp32.
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    batch, hk, keys = q.shape
    if normalize:
        q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6)
        k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    q = q * scale
    q = np.repeat(q, heads // hk, axis=1).astype(F32)
    k = np.repeat(k, heads // hk, axis=1).astype(F32)
    g = np.asarray(g, F32)
    beta = np.asarray(beta, F32)
    if a_log is not None:
        a_log = np.asarray(a_log, F32)
        bias = np.asarray(dt_bias, F32)
        if kda:
            u = g.reshape(batch, heads, keys) + bias.reshape(heads, keys)[None]
            g = (-np.exp(a_log)[None, :, None] * _softplus_gate(u)).astype(F32)
        else:
            u = g.reshape(batch, heads) + bias.reshape(heads)[None]
            g = (-np.exp(a_log)[None, :] * _softplus_gate(u)).astype(F32)
        beta = (1.0 / (1.0 + np.exp(-beta.astype(np.float64)))).astype(F32)
    return q, k, g, beta


def decode_step(pages, slots, plan: Plan, values, q, k, v, g, beta, storage="packed", **prep):
    """One packed-state decode step over ``pages[slots]`` (slot <= 0 = padding).

    Returns (out [B,H,V] fp32, new_pages copy, updated fp32 state [B,H,K,V]).
    """
    pages = np.array(pages, np.uint8)
    slots = np.asarray(slots).astype(np.int64)
    heads = plan.bits.shape[0]
    qp, kp, log_decay, beta_p = prepare_inputs(q, k, g, beta, heads, kda=plan.architecture == "kda", **prep)
    active = slots > 0
    state = np.zeros((len(slots), heads, plan.bits.shape[1], values), F32)
    if active.any():
        state[active] = page_decode(pages[slots[active]], plan, values, storage)
    out, updated = delta_step(state, qp, kp, np.asarray(v, F32).reshape(len(slots), heads, values),
                              log_decay, beta_p)
    out[~active] = 0
    if active.any():
        pages[slots[active]] = page_encode(updated[active], plan, pages[slots[active]], storage)
    return out, pages, updated


def row_impact(q, k, log_decay, beta):
    """core.py:18-24."""
    q, k = np.asarray(q, F32), np.asarray(k, F32)
    decay = np.exp(np.asarray(log_decay, F32))
    if decay.ndim == q.ndim - 1:
        decay = decay[..., None]
    b = np.asarray(beta, F32)[..., None]
    return np.square(decay * (q - b * k * (k * q).sum(-1, keepdims=True))).astype(F32)


def impact_factors(omega, gamma=0.25, floor=1e-20):
    """core.py:27-29."""
    log_w = np.log(np.maximum(np.asarray(omega, np.float64), floor)) * (gamma / 2)
    return np.exp(log_w - log_w.mean(-1, keepdims=True)).astype(F32)


def prefill_sequential(q, k, v, g, beta, cu_seqlens, initial_state=None, scale=None, normalize=True):
    """Token-by-token prefill recurrence of adapters.RecurrentKernel (adapters.py:36-60).

    q, k: [tokens, HK, K]; v: [tokens, H, V]; g (log decay), beta: [tokens, H];
    cu_seqlens: [N + 1] sequence boundaries; initial_state: [N, H, K, V] or None.
    q and k are L2 normalised (eps 1e-6) when ``normalize``, q is then scaled
    (default K^-0.5); value head h reads qk head h // (H / HK).  Each token is
    one core.delta_step.  Returns (out [tokens, H, V], final [N, H, K, V]).
    """
    q = np.asarray(q, F32)
    k = np.asarray(k, F32)
    v = np.asarray(v, F32)
    g = np.asarray(g, F32)
    beta = np.asarray(beta, F32)
    tokens, hk, keys = q.shape
    heads, values = v.shape[1], v.shape[2]
    scale = keys ** -0.5 if scale is None else scale
    if normalize:
        q = (q / np.sqrt((q.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)).astype(F32)
        k = (k / np.sqrt((k.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)).astype(F32)
    q = (q * F32(scale)).astype(F32)
    q = np.repeat(q, heads // hk, axis=1)
    k = np.repeat(k, heads // hk, axis=1)
    bounds = np.asarray(cu_seqlens, np.int64)
    out = np.zeros((tokens, heads, values), F32)
    finals = []
    for n in range(len(bounds) - 1):
        state = (np.zeros((1, heads, keys, values), F32) if initial_state is None
                 else np.asarray(initial_state, F32)[n:n + 1].copy())
        for t in range(bounds[n], bounds[n + 1]):
            y, state = delta_step(state, q[t:t + 1], k[t:t + 1], v[t:t + 1], g[t:t + 1], beta[t:t + 1])
            out[t] = y[0]
        finals.append(state[0])
    return out, np.stack(finals) if finals else np.zeros((0, heads, keys, values), F32)


# ---------------------------------------------------------------------------
# baseline state formats (stepquant/formats.py, kernels/format_pool.py)
# ---------------------------------------------------------------------------

def format_spec(name):
    """formats.py:28-44 get_format -> (kind, bits, group)."""
    import re
    if name == "fp32":
        return "fp32", 32, 32
    m = re.fullmatch(r"sym_int([468])_g128", name)
    if m:
        return "symmetric", int(m[1]), 128
    m = re.fullmatch(r"dsq_int([46])", name)
    if m:
        return "dsq", int(m[1]), 128
    raise ValueError(f"unknown state format: {name}")


def format_layout(heads, keys, values, kind, bits, group):
    """kernels/format_pool.py:9-27: (offsets, rows, columns, page_bytes) of a
    baseline-format page: each row's codes as one little-endian bitstream,
    then per row the symmetric groups' (fp16 scale, fp16 zero) or the DSQ fp16
    row scale, then per head the DSQ (fp16 column scale, fp16 zero) pairs."""
    offsets, rows, columns = [], [], []
    cursor = 0
    for _ in range(heads * keys):
        offsets.append(cursor)
        cursor += values * bits // 8
    cursor = (cursor + 3) // 4 * 4
    for _ in range(heads * keys):
        rows.append(-1 if kind == "fp32" else cursor)
        cursor += 0 if kind == "fp32" else (2 if kind == "dsq" else values // group * 4)
    cursor = (cursor + 3) // 4 * 4
    for _ in range(heads):
        columns.append(cursor)
        cursor += values * 4 if kind == "dsq" else 0
    return offsets, rows, columns, cursor


def group_fit(x, bits, group):
    """formats.py:51-66 (symmetric groupwise absmax): codes, scale, zero, recon."""
    x = np.asarray(x, F32)
    y = x.reshape(*x.shape[:-1], -1, group)
    limit = F32(2 ** (bits - 1) - 1)
    s = fp16_scale((np.abs(y).max(-1, keepdims=True) / limit).astype(F32))
    z = np.full_like(s, limit)
    q = (np.clip(np.rint((y / s).astype(F32)), -limit, limit) + z).astype(F32)
    return q.reshape(x.shape), s, z, ((q - z) * s).astype(F32).reshape(x.shape)


def dual_fit(x, bits, pivots=None):
    """formats.py:69-82 (Q-Mamba DSQ dual axis): codes, r, c, zero, recon.
    ``pivots`` (bool [H, K]) marks fp16 rows; the baseline pools have none."""
    x = np.asarray(x, F32)
    mask = np.ones(x.shape[1:3], bool)[None, :, :, None] if pivots is None else ~pivots[None, :, :, None]
    mean = (torch_inner_sum(np.abs(x))[..., None] / F32(x.shape[-1])).astype(F32)
    r = fp16_scale(np.sqrt(np.maximum(mean, F32(1e-20))))
    y = (x / r).astype(F32)
    levels = F32(2 ** (min(bits, 8) - 1) - 1)
    c = fp16_scale(np.where(mask, (np.abs(y) / levels).astype(F32), F32(0)).max(-2, keepdims=True))
    q = np.minimum(np.maximum(np.rint((y / c).astype(F32)), -levels), levels).astype(F32)
    recon = np.where(mask, ((r * c).astype(F32) * q).astype(F32), x.astype(np.float16).astype(F32))
    return (q + levels).astype(F32), r, c, np.zeros_like(c), recon


def _put_codes(page, off, codes, bits):
    stream = pack(np.asarray(codes, np.int64), bits)
    page[off:off + stream.size] = stream


def format_page_encode(state, name, pages=None):
    """One page per request of a baseline-format pool (format_pool.py encode,
    format_pool.py:64-75 store, formats.py:51-82): codes bit-packed per row, scales as fp16."""
    kind, bits, group = format_spec(name)
    state = np.asarray(state, F32)
    batch, heads, keys, values = state.shape
    offsets, rows, columns, page_bytes = format_layout(heads, keys, values, kind, bits, group)
    out = np.zeros((batch, page_bytes), np.uint8) if pages is None else np.array(pages, np.uint8)
    if kind == "symmetric":
        codes, s, z, _ = group_fit(state, bits, group)
    else:
        codes, r, c, _, _ = dual_fit(state, bits)
    for i in range(batch):
        page = out[i]
        for h in range(heads):
            for k in range(keys):
                row = h * keys + k
                _put_codes(page, offsets[row], codes[i, h, k], bits)
                if kind == "symmetric":
                    for g in range(values // group):
                        _put_half(page, rows[row] + 4 * g, s[i, h, k, g, 0])
                        _put_half(page, rows[row] + 4 * g + 2, z[i, h, k, g, 0])
                else:
                    _put_half(page, rows[row], r[i, h, k, 0])
            if kind == "dsq":
                for v in range(values):
                    _put_half(page, columns[h] + 4 * v, c[i, h, 0, v])
                    _put_half(page, columns[h] + 4 * v + 2, 0.0)
    return out


def format_page_decode(pages, name, heads, keys, values):
    """format_pool.py:77-128 read, formats.py:51-82: symmetric (code - zero) * scale; DSQ (r c)(code - levels)."""
    kind, bits, group = format_spec(name)
    pages = np.asarray(pages, np.uint8)
    offsets, rows, columns, _ = format_layout(heads, keys, values, kind, bits, group)
    out = np.zeros((pages.shape[0], heads, keys, values), F32)
    levels = F32(2 ** (bits - 1) - 1)
    for i in range(pages.shape[0]):
        page = pages[i]
        for h in range(heads):
            col = None
            if kind == "dsq":
                col = np.array([_get_half(page, columns[h] + 4 * v) for v in range(values)], np.float16).astype(F32)
            for k in range(keys):
                row = h * keys + k
                nbytes = values * bits // 8
                codes = unpack(page[offsets[row]:offsets[row] + nbytes], bits, values).astype(F32)
                if kind == "symmetric":
                    s = np.repeat(np.array([_get_half(page, rows[row] + 4 * g) for g in range(values // group)],
                                           np.float16).astype(F32), group)
                    z = np.repeat(np.array([_get_half(page, rows[row] + 4 * g + 2) for g in range(values // group)],
                                           np.float16).astype(F32), group)
                    out[i, h, k] = ((codes - z).astype(F32) * s).astype(F32)
                else:
                    rr = np.float16(_get_half(page, rows[row])).astype(F32)
                    out[i, h, k] = ((rr * col).astype(F32) * (codes - levels).astype(F32)).astype(F32)
    return out
