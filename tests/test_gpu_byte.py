"""Byte-carrier pages (PackedStatePool(storage='byte'), kernels/pool.py:29-43,
fit.py:111-115, byte_codec.py:6-27) on the device against the oracle.

* encode writes exactly the oracle's byte-carrier page image (GDN heads of
  widths 4/6/8, a 2-bit head with value-group row scales and an fp16 pivot
  head; KDA heads of mixed row widths with pivot rows and an all-pivot head);
* decode reads back the oracle's dense state;
* a fused step repacks exactly the oracle's fit of the kernel's own updated
  state, the readout matches the oracle's; async (readout + writeback) pages
  equal fused pages.
"""
import numpy as np
import pytest
import torch

from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def _plan(arch, seed):
    from stepquant_b200 import QuantizationPlan
    gen = torch.Generator().manual_seed(seed)
    if arch == "gdn":
        bits = torch.tensor([4, 6, 8, 2, 16, 6])[:, None].expand(6, 128).clone()
    else:
        bits = torch.tensor([2, 4, 6, 16])[torch.randint(0, 4, (4, 128), generator=gen)]
        bits[3] = 16  # all-pivot head
    impact = torch.rand(bits.shape, generator=gen) + 0.25
    return (QuantizationPlan(arch, bits.cuda(), impact.cuda(), 32),
            O.Plan(arch, bits.numpy(), impact.numpy(), 32))


def _inputs(arch, batch, heads, gen):
    q = torch.randn(batch, heads, 128, generator=gen)
    k = torch.randn(batch, heads, 128, generator=gen)
    v = torch.randn(batch, heads, 128, generator=gen)
    a = torch.randn(batch, heads, 128, generator=gen) if arch == "kda" else torch.randn(batch, heads, generator=gen)
    b = torch.randn(batch, heads, generator=gen)
    return q, k, v, a, b


@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_byte_pages_encode_decode_step(arch):
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(31)
    plan, oplan = _plan(arch, 31)
    heads, batch = plan.bits.shape[0], 5
    pool = PackedStatePool(plan, batch + 1, 128, storage="byte")
    assert pool.page_bytes == O.packed_layout(oplan, 128, "byte")[-1]
    slots = torch.tensor([2, 5, 0, 1, 4], device="cuda")
    state = torch.randn(batch, heads, 128, 128, generator=gen) * 0.1
    pool.encode(state.cuda(), slots)
    pool.check_status()
    pages = pool.data.cpu().numpy()
    s = slots.cpu().numpy()
    active = s > 0
    expected = O.page_encode(state.numpy()[active], oplan, storage="byte")
    for j, slot in enumerate(s[active]):
        assert (pages[slot] == expected[j]).all(), f"encode, slot {slot}"
    dense = pool.decode(slots).cpu().numpy()
    np.testing.assert_array_equal(dense[active], O.page_decode(expected, oplan, 128, "byte"))

    q, k, v, a, b = _inputs(arch, batch, heads, gen)
    a_log = torch.rand(heads) * np.log(16)
    dt_bias = torch.zeros(heads * 128 if arch == "kda" else heads)
    kw = dict(normalize=True, scale=128 ** -0.5)
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    before = pool.data.cpu().numpy()
    out = pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, a_log=a_log.cuda(), dt_bias=dt_bias.cuda(),
                    state_out=upd, **kw)
    pool.check_status()
    o_out, _, o_upd = O.decode_step(before, s, oplan, 128, q.numpy(), k.numpy(), v.numpy(), a.numpy(), b.numpy(),
                                    storage="byte", a_log=a_log.numpy(), dt_bias=dt_bias.numpy(), **kw)
    u = upd.cpu().numpy()
    assert np.abs(u[active] - o_upd[active]).max() <= 1e-3 * np.abs(o_upd).max()
    np.testing.assert_allclose(out.cpu().numpy(), o_out, atol=5e-5, rtol=1e-4)
    expected = O.page_encode(u[active], oplan, before[s[active]], storage="byte")
    pages = pool.data.cpu().numpy()
    for j, slot in enumerate(s[active]):
        assert (pages[slot] == expected[j]).all(), f"step, slot {slot}"
    assert (pages[3] == before[3]).all()  # slot 3 is not in this batch


@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_byte_pages_async_equals_fused(arch):
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(37)
    plan, _ = _plan(arch, 37)
    heads, batch = plan.bits.shape[0], 7
    sync = PackedStatePool(plan, batch + 1, 128, storage="byte")
    asyn = PackedStatePool(plan, batch + 1, 128, writeback_stream=torch.cuda.Stream(), storage="byte")
    slots = torch.arange(1, batch + 1, device="cuda")
    state = torch.randn(batch, heads, 128, 128, generator=gen).cuda() * 0.1
    sync.encode(state, slots)
    asyn.encode(state, slots)
    a_log = torch.rand(heads).cuda()
    dt_bias = torch.zeros(heads * 128 if arch == "kda" else heads).cuda()
    for step in range(3):
        q, k, v, a, b = (t.cuda().bfloat16() if i < 3 else t.cuda()
                         for i, t in enumerate(_inputs(arch, batch, heads, gen)))
        o1 = sync.step(q, k, v, a, b, slots, normalize=True, scale=128 ** -0.5, a_log=a_log, dt_bias=dt_bias)
        o2 = asyn.step(q, k, v, a, b, slots, normalize=True, scale=128 ** -0.5, a_log=a_log, dt_bias=dt_bias)
        asyn.wait()
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        assert torch.equal(sync.data, asyn.data), f"step {step}"
