"""GDN 2-bit heads on their own kernel (csrc/sq_fast_two.cu) against the oracle.

The reference's Qwen INT2 rows (quantization.py:69-87): levels {-3,-1,1,3},
an fp16 row scale per 32-value group, the group |x| sums in torch's order.

* encode: page bytes == the oracle's page image (also with rows beyond 2^96,
  the IEEE-division path), decode == the oracle's page decode;
* fused step: repacked bytes == the oracle's fit_state of the kernel's own
  updated state, readout within the usual tolerances;
* asynchronous readout + writeback == fused bytes and outputs, over three
  steps, at a batch where every SM runs many 2-bit items.
"""
import numpy as np
import pytest
import torch

from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def _plan(widths, seed):
    from stepquant_b200 import QuantizationPlan
    gen = torch.Generator().manual_seed(seed)
    heads = len(widths)
    bits = torch.tensor(widths)[:, None].expand(heads, 128).clone()
    impact = torch.rand(heads, 128, generator=gen) + 0.25
    return QuantizationPlan("gdn", bits.cuda(), impact.cuda()), O.Plan("gdn", bits.numpy(), impact.numpy())


def _inputs(batch, heads, qk_heads, gen, dtype=torch.bfloat16):
    q = torch.randn(batch, qk_heads, 128, generator=gen).to(dtype)
    k = torch.randn(batch, qk_heads, 128, generator=gen).to(dtype)
    v = torch.randn(batch, heads, 128, generator=gen).to(dtype)
    a = torch.randn(batch, heads, generator=gen)
    b = torch.randn(batch, heads, generator=gen)
    return q, k, v, a, b


MIXED = [2, 4, 2, 8, 16, 2, 6, 2]


def test_two_bit_encode_decode_match_oracle():
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(21)
    plan, oplan = _plan(MIXED, 21)
    batch, heads = 10, len(MIXED)
    pool = PackedStatePool(plan, batch + 1, 128)
    slots = torch.arange(1, batch + 1, device="cuda")
    state = torch.randn(batch, heads, 128, 128, generator=gen) * 0.1
    state[2] *= 40.0
    state[4, 0, 3] *= 1e29  # a 2-bit head's group sums beyond 2^96: the IEEE-division path
    before = pool.data.cpu().numpy()
    pool.encode(state.cuda(), slots)
    pool.check_status()
    got = pool.data.cpu().numpy()
    expected = O.page_encode(state.numpy(), oplan, before[1:])
    for i in range(batch):
        assert (got[1 + i] == expected[i]).all(), f"request {i}: page bytes differ"
    assert (got[0] == before[0]).all()
    dense = pool.decode(slots).cpu().numpy()
    ref = O.page_decode(got[1:], oplan, 128)
    assert np.array_equal(dense, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_two_bit_step_matches_oracle(dtype):
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(22)
    plan, oplan = _plan(MIXED, 22)
    batch, heads, qk = 48, len(MIXED), 4
    pool = PackedStatePool(plan, batch + 1, 128)
    slots = torch.arange(1, batch + 1, device="cuda")
    slots[5] = 0
    pool.encode(torch.randn(batch, heads, 128, 128, device="cuda") * 0.1, slots)
    a_log, dt_bias = torch.rand(heads) * np.log(16), torch.zeros(heads)
    q, k, v, a, b = _inputs(batch, heads, qk, gen, dtype)
    before = pool.data.cpu().numpy()
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    out = pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, normalize=True, scale=128 ** -0.5,
                    a_log=a_log.cuda(), dt_bias=dt_bias.cuda(), state_out=upd)
    pool.check_status()
    pages = pool.data.cpu().numpy()
    s = slots.cpu().numpy()
    check = [0, 1, 6, 30, 47]
    o_out, _, o_upd = O.decode_step(before, s[check], oplan, 128, q[check].float().numpy(), k[check].float().numpy(),
                                    v[check].float().numpy(), a[check].numpy(), b[check].numpy(), normalize=True,
                                    scale=128 ** -0.5, a_log=a_log.numpy(), dt_bias=dt_bias.numpy())
    u = upd.cpu().numpy()
    assert np.abs(u[check] - o_upd).max() <= 1e-3 * np.abs(o_upd).max()
    tol = dict(atol=5e-5, rtol=1e-4) if dtype == torch.float32 else dict(atol=2e-2, rtol=0)
    np.testing.assert_allclose(out.float().cpu().numpy()[check], o_out, **tol)
    expected = O.page_encode(u[check], oplan, before[s[check]])
    for j, i in enumerate(check):
        assert (pages[s[i]] == expected[j]).all(), f"request {i}: packed bytes differ"
    assert out[5].count_nonzero() == 0 and (pages[0] == before[0]).all()


def test_two_bit_async_equals_fused():
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(23)
    widths = [2] * 12 + [4] * 4 + [6] * 8 + [8] * 8
    widths = [widths[i] for i in torch.randperm(32, generator=gen).tolist()]
    plan, oplan = _plan(widths, 23)
    batch, heads, qk = 256, 32, 16
    sync = PackedStatePool(plan, batch + 1, 128)
    asyn = PackedStatePool(plan, batch + 1, 128, writeback_stream=torch.cuda.Stream(), writeback_chunk=0)
    slots = torch.randperm(batch, generator=gen).cuda() + 1
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.1
    sync.encode(state, slots)
    asyn.encode(state, slots)
    assert torch.equal(sync.data, asyn.data)
    kw = dict(normalize=True, scale=128 ** -0.5, a_log=(torch.rand(heads) * np.log(16)).cuda(),
              dt_bias=torch.zeros(heads).cuda())
    for step in range(3):
        q, k, v, a, b = (t.cuda() for t in _inputs(batch, heads, qk, gen))
        before = sync.data.cpu().numpy()
        upd = torch.empty(batch, heads, 128, 128, device="cuda")
        o1 = sync.step(q, k, v, a, b, slots, state_out=upd, **kw)
        o2 = asyn.step(q, k, v, a, b, slots, **kw)
        asyn.wait()
        torch.cuda.synchronize()
        sync.check_status()
        asyn.check_status()
        assert torch.equal(o1, o2), f"step {step}: readout differs"
        assert torch.equal(sync.data, asyn.data), f"step {step}: pages differ"
        s = slots.cpu().numpy()
        pick = [0, 77, 255]
        expected = O.page_encode(upd.cpu().numpy()[pick], oplan, before[s[pick]])
        got = sync.data.cpu().numpy()
        for j, i in enumerate(pick):
            assert (got[s[i]] == expected[j]).all(), f"step {step}, request {i}"
