"""Little-endian bit packing on the device (the reference's ``stepquant.packing``, packing.py:6-22).

``pack(codes, bits)``: n = 8/gcd(bits, 8) codes in n*bits/8 bytes, code i at
bit offset i*bits.  CUDA tensors only (``sq_pack`` / ``sq_unpack``).  The
reference's widths are 2, 4, 6 and 8; ``extended=True`` also admits this
package's 3- and 5-bit extension (8 codes in 3 or 5 bytes).
"""
import torch

from . import _native as N


def _check(bits, extended):
    if bits not in ((2, 3, 4, 5, 6, 8) if extended else (2, 4, 6, 8)):
        raise ValueError("supported code widths: 2, 4, 6, 8")


def pack(codes, bits, extended=False):
    _check(bits, extended)
    N.require_cuda(codes)
    flat = codes.reshape(-1).to(torch.int16).contiguous()
    out = torch.empty(int(N.lib().sq_packed_bytes(flat.numel(), bits)), device=codes.device, dtype=torch.uint8)
    N.check(N.lib().sq_pack(N.ptr(flat), flat.numel(), bits, N.ptr(out), N.stream_handle()))
    return out


def unpack(data, bits, count, extended=False):
    _check(bits, extended)
    N.require_cuda(data)
    data = data.reshape(-1).contiguous()
    if int(N.lib().sq_packed_bytes(count, bits)) > data.numel():
        raise ValueError("packed stream is shorter than count codes")
    out = torch.empty(count, device=data.device, dtype=torch.int16)
    N.check(N.lib().sq_unpack(N.ptr(data), count, bits, N.ptr(out), N.stream_handle()))
    return out
