"""sq_step_async_noalloc against the allocating asynchronous step, through the C ABI.

Callers that cannot allocate device memory while they step (a server that
reserves its whole device budget at start-up, or a binding with no device
allocator of its own) use sq_step_async_noalloc, whose scratch is a fixed
file-scope device array of the library.  Its output and repacked pages must
match sq_readout + sq_writeback with caller-allocated scratch: outputs within
the readout tolerance used by the other tests (atol 5e-5, rtol 1e-4; they are
in fact expected to be equal) and page bytes identical, on two calls in a row.

This file is named to be collected last: a failure here leaves every other
test already run.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(batch, heads=6, qk_heads=3, keys=128, values=128, seed=11):
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.quantization import DevicePlan
    torch.manual_seed(seed)
    bits = torch.tensor([4, 6, 8, 16, 2, 6])[:heads, None].expand(heads, keys).clone()
    plan = QuantizationPlan("gdn", bits.cuda(), (torch.rand(heads, keys) + 0.5).cuda())
    dp = DevicePlan(plan, values)
    num_slots = batch + 2
    pages = torch.zeros(num_slots, dp.page_bytes, device="cuda", dtype=torch.uint8)
    return plan, dp, pages, num_slots


def _args(N, q, k, v, g, b, a_log, dt_bias, out, qk_heads, keys):
    return N.SqStepArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), k.stride(0), v.stride(0), qk_heads,
                        N.dtype_code(q.dtype), g.data_ptr(), b.data_ptr(), N.SQ_F32, 1, a_log.data_ptr(),
                        dt_bias.data_ptr(), keys ** -0.5, 0, out.data_ptr())


def test_noalloc_step_matches_allocating_step_on_two_calls():
    from stepquant_b200 import _native as N
    lib = N.lib()
    batch, heads, qk_heads, keys, values = 7, 6, 3, 128, 128
    plan, dp, pages_a, num_slots = _setup(batch, heads, qk_heads, keys, values)
    slots = torch.tensor([3, 1, 0, 5, 2, 8, 4], device="cuda", dtype=torch.int64)
    state = torch.randn(batch, heads, keys, values, device="cuda") * 0.1
    status = torch.zeros(1, device="cuda", dtype=torch.int32)
    stream = N.stream_handle()
    N.check(lib.sq_encode(dp.ref(), N.ptr(state), N.ptr(slots), batch, N.ptr(pages_a), num_slots, N.ptr(status),
                          stream))
    pages_b = pages_a.clone()
    floats = lib.sq_scratch_floats(dp.ref())
    scratch = torch.empty(batch, floats, device="cuda")
    stable = torch.empty(batch, device="cuda", dtype=torch.int64)
    a_log = torch.rand(heads, device="cuda")
    dt_bias = torch.zeros(heads, device="cuda")
    for call in range(2):
        q = torch.randn(batch, qk_heads, keys, device="cuda", dtype=torch.bfloat16)
        k = torch.randn_like(q)
        v = torch.randn(batch, heads, values, device="cuda", dtype=torch.bfloat16)
        g = torch.randn(batch, heads, device="cuda")
        b = torch.randn(batch, heads, device="cuda")
        out_a = torch.empty(batch, heads, values, device="cuda", dtype=torch.bfloat16)
        out_b = torch.empty_like(out_a)
        args_a = _args(N, q, k, v, g, b, a_log, dt_bias, out_a, qk_heads, keys)
        args_b = _args(N, q, k, v, g, b, a_log, dt_bias, out_b, qk_heads, keys)
        N.check(lib.sq_readout(dp.ref(), N.ptr(pages_a), num_slots, N.ptr(slots), batch, ctypes.byref(args_a),
                               N.ptr(scratch), N.ptr(stable), N.ptr(status), stream))
        N.check(lib.sq_writeback(dp.ref(), N.ptr(pages_a), num_slots, N.ptr(stable), batch, N.ptr(scratch), None,
                                 N.ptr(status), stream))
        N.check(lib.sq_step_async_noalloc(dp.ref(), N.ptr(pages_b), num_slots, N.ptr(slots), batch,
                                          ctypes.byref(args_b), N.ptr(status), stream))
        torch.cuda.synchronize()
        torch.testing.assert_close(out_b.float(), out_a.float(), atol=5e-5, rtol=1e-4)
        assert torch.equal(pages_b, pages_a), f"call {call}: repacked pages differ"
        assert out_b[2].count_nonzero() == 0
    assert int(status.item()) == 0


def test_noalloc_step_rejects_batches_beyond_its_array():
    from stepquant_b200 import _native as N
    lib = N.lib()
    _, dp, pages, num_slots = _setup(2)
    floats = lib.sq_scratch_floats(dp.ref())
    limit = lib.sq_noalloc_scratch_bytes()
    too_many = int(limit // (floats * 4)) + 1
    x = torch.zeros(1, device="cuda")
    args = N.SqStepArgs(x.data_ptr(), x.data_ptr(), x.data_ptr(), 0, 0, 0, 6, N.SQ_F32, x.data_ptr(), x.data_ptr(),
                        N.SQ_F32, 0, None, None, 1.0, 0, x.data_ptr())
    code = lib.sq_step_async_noalloc(dp.ref(), N.ptr(pages), num_slots, N.ptr(x), too_many, ctypes.byref(args),
                                     None, N.stream_handle())
    assert code == N.SQ_ERR_CAPACITY
    with pytest.raises(ValueError, match="capacity"):
        N.check(code)
