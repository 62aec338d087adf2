"""Register-resident K = V = 128 KDA kernels (csrc/sq_fast_kda.cu) against the oracle.

* a full step repacks bit-exactly what the oracle's fit_state gives for the
  kernel's own pre-quantization state (per-row widths {2, 4, 6, 8}, fp16 pivot
  rows), readout within atol 5e-5 / rtol 1e-4 (fp32 out) and 2e-2 (bf16 out);
* heads the kernel leaves to the tile kernel (a code region larger than its
  stage buffer, an all-pivot head) are handled in the same launch;
* async (readout + writeback) bytes == fused bytes over several steps.
"""
import numpy as np
import pytest
import torch

from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def _kda_plan(heads, seed, extra=()):
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200 import synthetic as S
    gen = torch.Generator().manual_seed(seed)
    bits = S.kda_widths(heads, 128, gen, choices=(2, 4, 6, 8), probs=(0.3, 0.4, 0.2, 0.1))
    for h, kind in extra:
        if kind == "wide":      # mostly pivots: code region beyond the fast kernel's stage
            bits[h] = 16
            bits[h, :3] = 4
        elif kind == "pivot":   # all-pivot head
            bits[h] = 16
    impact = torch.rand(heads, 128, generator=gen) + 0.25
    return QuantizationPlan("kda", bits.cuda(), impact.cuda()), O.Plan("kda", bits.numpy(), impact.numpy())


def _inputs(batch, heads, gen, dtype):
    q = torch.randn(batch, heads, 128, generator=gen).to(dtype)
    k = torch.randn(batch, heads, 128, generator=gen).to(dtype)
    v = torch.randn(batch, heads, 128, generator=gen).to(dtype)
    a = torch.randn(batch, heads, 128, generator=gen)
    b = torch.randn(batch, heads, generator=gen)
    return q, k, v, a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_kda_step_bytes_exact_and_readout(dtype):
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(21)
    heads, batch = 8, 48
    plan, oplan = _kda_plan(heads, 21, extra=((5, "wide"), (6, "pivot")))
    pool = PackedStatePool(plan, batch + 1, 128)
    slots = torch.arange(1, batch + 1, device="cuda")
    slots[7] = 0
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.1
    pool.encode(state, slots)
    a_log = torch.rand(heads) * np.log(16)
    dt_bias = torch.randn(heads * 128) * 0.1
    q, k, v, a, b = _inputs(batch, heads, gen, dtype)
    before = pool.data.cpu().numpy()
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    out = pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, normalize=True, scale=128 ** -0.5,
                    a_log=a_log.cuda(), dt_bias=dt_bias.cuda(), state_out=upd)
    pool.check_status()
    pages = pool.data.cpu().numpy()
    s = slots.cpu().numpy()
    check = [0, 1, 20, 47]
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
    assert out[7].count_nonzero() == 0 and (pages[0] == before[0]).all()
    # Every request: the step's bytes equal the tile encoder's for its own state.
    pool2 = PackedStatePool(plan, batch + 1, 128)
    active = slots > 0
    pool2.data.copy_(pool.data)
    pool2.encode(upd[active], slots[active])
    assert torch.equal(pool2.data, pool.data)


def test_kda_async_equals_fused():
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(23)
    heads, batch = 6, 40
    plan, _ = _kda_plan(heads, 23, extra=((2, "wide"),))
    sync = PackedStatePool(plan, batch + 2, 128)
    asyn = PackedStatePool(plan, batch + 2, 128, writeback_stream=torch.cuda.Stream())
    slots = torch.randperm(batch + 1, generator=gen)[:batch].cuda() + 1
    slots[3] = 0
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.2
    sync.encode(state, slots)
    asyn.encode(state, slots)
    a_log, dt_bias = torch.rand(heads).cuda(), torch.zeros(heads * 128).cuda()
    for step in range(3):
        q, k, v, a, b = (t.cuda() for t in _inputs(batch, heads, gen, torch.bfloat16))
        o1 = sync.step(q, k, v, a, b, slots, normalize=True, scale=128 ** -0.5, a_log=a_log, dt_bias=dt_bias)
        o2 = asyn.step(q, k, v, a, b, slots, normalize=True, scale=128 ** -0.5, a_log=a_log, dt_bias=dt_bias)
        asyn.wait()
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        assert torch.equal(sync.data, asyn.data), f"step {step}"


def test_kda_saturated_scales():
    """A state with integer rows near 1e27 encodes to saturated fp16 scales
    (r, c = 65504); the KDA kernel's step from those pages repacks exactly the
    oracle's fit_state of its own updated state."""
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(24)
    heads, batch = 4, 6
    plan, oplan = _kda_plan(heads, 24)
    pool = PackedStatePool(plan, batch + 1, 128)
    slots = torch.arange(1, batch + 1, device="cuda")
    state = torch.randn(batch, heads, 128, 128, generator=gen) * 0.1
    bits = oplan.bits
    rows = [k for k in range(128) if bits[1, k] != 16][:2]
    state[2, 1, rows] *= 1e28
    pool.encode(state.cuda(), slots)
    q, k, v, a, b = _inputs(batch, heads, gen, torch.float32)
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    before = pool.data.cpu().numpy()
    pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, normalize=True, scale=128 ** -0.5,
              a_log=(torch.rand(heads) * np.log(16)).cuda(), dt_bias=torch.zeros(heads * 128).cuda(), state_out=upd)
    pool.check_status()
    u = upd.cpu().numpy()
    assert np.isfinite(u).all() and np.abs(u).max() > 1e6
    expected = O.page_encode(u, oplan, before[1:])
    got = pool.data.cpu().numpy()
    for i in range(batch):
        assert (got[i + 1] == expected[i]).all(), f"request {i}"
