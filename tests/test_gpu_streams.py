"""SM-budget writeback streams (``writeback_resources``, csrc/sq_streams.cu).

A budgeted stream is a green-context stream holding at least the requested
SMs; the persistent writeback kernel sizes its grid to those SMs, so with a
16-SM budget each CTA takes several items.  The bytes written from such a
stream equal the fused step's.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_budget_stream_writeback_equals_fused():
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.resources import writeback_resources
    res = writeback_resources("cuda", 16)
    assert 16 <= res.actual_sms < res.total_sms and res.requested_sms == 16
    assert writeback_resources(torch.device("cuda"), 16) is res
    assert writeback_resources("cuda", 0).actual_sms == res.total_sms
    with pytest.raises(ValueError):
        writeback_resources("cuda", res.total_sms + 1)
    gen = torch.Generator().manual_seed(31)
    heads, batch = 4, 96
    bits = torch.tensor([4, 6, 8, 6])[:, None].expand(heads, 128).clone()
    plan = QuantizationPlan("gdn", bits.cuda(), (torch.rand(heads, 128, generator=gen) + 0.25).cuda())
    sync = PackedStatePool(plan, batch + 1, 128)
    asyn = PackedStatePool(plan, batch + 1, 128, writeback_stream=res.stream)
    slots = torch.randperm(batch, generator=gen).cuda() + 1
    state = torch.randn(batch, heads, 128, 128, generator=gen).cuda() * 0.1
    sync.encode(state, slots)
    asyn.encode(state, slots)
    kw = dict(normalize=True, scale=128 ** -0.5, a_log=torch.rand(heads).cuda(), dt_bias=torch.zeros(heads).cuda())
    for step in range(2):
        q, k, v = (torch.randn(batch, heads, 128, generator=gen).bfloat16().cuda() for _ in range(3))
        a, b = (torch.randn(batch, heads, generator=gen).cuda() for _ in range(2))
        o1 = sync.step(q, k, v, a, b, slots, **kw)
        o2 = asyn.step(q, k, v, a, b, slots, **kw)
        asyn.wait()
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        assert torch.equal(sync.data, asyn.data), f"step {step}"
