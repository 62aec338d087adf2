"""ctypes binding of libstepquant_b200.so (the C ABI in include/stepquant_b200.h).

The library is built in-tree by ``stepquant_b200._build``.  There is no
fallback: if the library is missing every device operation raises.
"""
import ctypes
import os

import torch

from ._build import LIBRARY

SQ_OK, SQ_ERR_ARGUMENT, SQ_ERR_SHAPE, SQ_ERR_UNSUPPORTED, SQ_ERR_CUDA, SQ_ERR_CAPACITY = range(6)
SQ_STATUS_SLOT_RANGE = 1
SQ_STATUS_TIMEOUT = 2
SQ_F32, SQ_BF16, SQ_F16 = 0, 1, 2
SQ_GDN, SQ_KDA = 0, 1

_DTYPES = {torch.float32: SQ_F32, torch.bfloat16: SQ_BF16, torch.float16: SQ_F16}

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class SqPlan(ctypes.Structure):
    _fields_ = [("architecture", _i32), ("heads", _i32), ("keys", _i32), ("values", _i32),
                ("value_group_size", _i32), ("storage", _i32), ("page_bytes", _i64),
                ("bits", _p), ("impact", _p), ("offsets", _p), ("rows", _p), ("columns", _p),
                ("bits_host", _p)]


class SqStepArgs(ctypes.Structure):
    _fields_ = [("q", _p), ("k", _p), ("v", _p), ("q_stride", _i64), ("k_stride", _i64), ("v_stride", _i64),
                ("qk_heads", _i32), ("io_dtype", _i32), ("g", _p), ("beta", _p), ("gate_dtype", _i32),
                ("normalize", _i32), ("a_log", _p), ("dt_bias", _p), ("scale", ctypes.c_float),
                ("reserved", _i32), ("out", _p)]


class SqPrefillArgs(ctypes.Structure):
    _fields_ = [("q", _p), ("k", _p), ("v", _p), ("q_stride", _i64), ("k_stride", _i64), ("v_stride", _i64),
                ("io_dtype", _i32), ("qk_heads", _i32), ("heads", _i32), ("keys", _i32), ("values", _i32),
                ("normalize", _i32), ("scale", ctypes.c_float), ("num_seqs", _i32), ("tokens", _i32), ("cu_seqlens", _p),
                ("g", _p), ("beta", _p), ("initial_state", _p), ("final_state", _p), ("out", _p),
                ("workspace", _p), ("workspace_bytes", _i64), ("status", _p)]


_SIGNATURES = {
    "sq_version": (_i32, []),
    "sq_error_string": (ctypes.c_char_p, [_i32]),
    "sq_packed_layout": (_i32, [_i32, _i32, _i32, _i32, _i32, _p, _i32, _p, _p, _p, _p]),
    "sq_encode": (_i32, [_p, _p, _p, _i32, _p, _i64, _p, _p]),
    "sq_decode": (_i32, [_p, _p, _i64, _p, _i32, _p, _p, _p]),
    "sq_step": (_i32, [_p, _p, _i64, _p, _i32, _p, _p, _p, _p]),
    "sq_scratch_floats": (_i64, [_p]),
    "sq_readout": (_i32, [_p, _p, _i64, _p, _i32, _p, _p, _p, _p, _p]),
    "sq_writeback": (_i32, [_p, _p, _i64, _p, _i32, _p, _p, _p, _p]),
    "sq_fit_state": (_i32, [_p, _p, _i32, _p, _p, _p, _p, _p, _p]),
    "sq_pack": (_i32, [_p, _i64, _i32, _p, _p]),
    "sq_packed_bytes": (_i64, [_i64, _i32]),
    "sq_unpack": (_i32, [_p, _i64, _i32, _p, _p]),
    "sq_fp32_step": (_i32, [_p, _i64, _i32, _i32, _i32, _i32, _p, _i32, _p, _p, _p]),
    "sq_step_async_noalloc": (_i32, [_p, _p, _i64, _p, _i32, _p, _p, _p]),
    "sq_noalloc_scratch_bytes": (_i64, []),
    "sq_budget_stream": (_i32, [_i32, _i32, ctypes.POINTER(_p), ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "sq_selftest_fp16_division": (_i32, [_p, _p, _p, _i64, _p]),
    "sq_gdn_prefill": (_i32, [_p, _p]),
    "sq_gdn_prefill_workspace_bytes": (_i64, [_i32, _i32, _i32]),
    "sq_kda_prefill": (_i32, [_p, _p]),
}

EXPORTED = tuple(_SIGNATURES)
_lib = None


def library_path():
    return LIBRARY


def lib():
    """The loaded library; raises RuntimeError when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY):
            raise RuntimeError(
                f"stepquant_b200 native library not found at {LIBRARY}; build it with "
                "`python -m stepquant_b200._build` (there is no CPU fallback)")
        handle = ctypes.CDLL(LIBRARY)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


class NativeError(RuntimeError):
    pass


def check(code):
    """Map an sq_error code to the reference's exception types."""
    if code == SQ_OK:
        return
    text = lib().sq_error_string(code).decode()
    if code in (SQ_ERR_ARGUMENT, SQ_ERR_SHAPE, SQ_ERR_CAPACITY):
        raise ValueError(f"stepquant_b200: {text}")
    if code == SQ_ERR_UNSUPPORTED:
        raise NotImplementedError(f"stepquant_b200: {text}")
    raise NativeError(f"stepquant_b200: {text} ({torch.cuda.get_device_name() if torch.cuda.is_available() else 'no device'})")


def dtype_code(dtype):
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; use float32, bfloat16 or float16") from None


def ptr(tensor):
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def stream_handle(stream=None):
    stream = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(stream.cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError("stepquant_b200 operates on CUDA tensors only (no CPU fallback)")
