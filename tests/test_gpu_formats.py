"""Baseline-format pools (FormatStatePool: sym_int4/6/8_g128, dsq_int4/6;
kernels/format_pool.py) on the device against the oracle.

* encode writes exactly the oracle's page image (codes and fp16 scales of the
  reference's ``group_fit`` / ``dual_fit``, pinned by tests/golden/formats.npz);
* decode returns the oracle's reconstruction bit for bit;
* a step's readout and updated state match the oracle's delta rule on the
  decoded state, and its pages are exactly the format fit of the kernel's
  own updated state.
"""
import numpy as np
import pytest
import torch

from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu

NAMES = ["sym_int4_g128", "sym_int6_g128", "sym_int8_g128", "dsq_int4", "dsq_int6"]


def _pool(name, arch, heads, keys, values, slots, seed):
    from stepquant_b200.formats import get_format
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.format_pool import FormatStatePool
    spec = get_format(name)
    gen = torch.Generator().manual_seed(seed)
    bits = torch.full((heads, keys), spec.bits, dtype=torch.long)
    plan = QuantizationPlan(arch, bits.cuda(), (torch.rand(heads, keys, generator=gen) + 0.5).cuda())
    return FormatStatePool(plan, slots, values, spec), gen


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_format_pool_encode_decode_step(name, arch):
    heads, keys, values, batch = 4, 64, 128, 5
    pool, gen = _pool(name, arch, heads, keys, values, batch + 1, 51)
    kind, bits, group = O.format_spec(name)
    assert pool.page_bytes == O.format_layout(heads, keys, values, kind, bits, group)[-1]
    slots = torch.tensor([3, 1, 0, 5, 2], device="cuda")
    s = slots.cpu().numpy()
    active = s > 0
    state = torch.randn(batch, heads, keys, values, generator=gen) * 0.1
    state[1, 2, 7] = 0  # an all-zero row
    pool.encode(state.cuda(), slots)
    pool.check_status()
    pages = pool.data.cpu().numpy()
    expected = O.format_page_encode(state.numpy()[active], name)
    for j, slot in enumerate(s[active]):
        assert (pages[slot] == expected[j]).all(), f"encode, slot {slot}"
    recon = O.format_page_decode(expected, name, heads, keys, values)
    np.testing.assert_array_equal(pool.decode(slots).cpu().numpy()[active], recon)

    q = torch.randn(batch, heads, keys, generator=gen)
    k = torch.randn(batch, heads, keys, generator=gen)
    v = torch.randn(batch, heads, values, generator=gen)
    a = torch.randn(batch, heads, keys, generator=gen) if arch == "kda" else torch.randn(batch, heads, generator=gen)
    b = torch.randn(batch, heads, generator=gen)
    a_log = torch.rand(heads) * np.log(16)
    dt_bias = torch.zeros(heads * keys if arch == "kda" else heads)
    upd = torch.empty(batch, heads, keys, values, device="cuda")
    out = pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, normalize=True, scale=keys ** -0.5,
                    a_log=a_log.cuda(), dt_bias=dt_bias.cuda(), state_out=upd)
    pool.check_status()
    qp, kp, g, beta = O.prepare_inputs(q.numpy(), k.numpy(), a.numpy(), b.numpy(), heads, kda=arch == "kda",
                                       normalize=True, scale=keys ** -0.5, a_log=a_log.numpy(), dt_bias=dt_bias.numpy())
    o_out, o_upd = O.delta_step(recon, qp[active], kp[active], v.numpy()[active], g[active], beta[active])
    u = upd.cpu().numpy()
    assert np.abs(u[active] - o_upd).max() <= 1e-3 * np.abs(o_upd).max()
    np.testing.assert_allclose(out.cpu().numpy()[active], o_out, atol=5e-5, rtol=1e-4)
    assert out[~torch.from_numpy(active)].count_nonzero() == 0
    expected = O.format_page_encode(u[active], name)
    pages = pool.data.cpu().numpy()
    for j, slot in enumerate(s[active]):
        assert (pages[slot] == expected[j]).all(), f"step, slot {slot}"


def test_format_pool_validation():
    from stepquant_b200.formats import get_format
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.format_pool import Fp32StatePool, FormatStatePool
    bits = torch.full((2, 32), 4, dtype=torch.long).cuda()
    plan = QuantizationPlan("gdn", bits, torch.ones(2, 32).cuda())
    with pytest.raises(ValueError):  # precision map differs from the format's width
        FormatStatePool(plan, 3, 128, get_format("sym_int8_g128"))
    with pytest.raises(ValueError):  # the fused formats are synchronous
        FormatStatePool(plan, 3, 128, get_format("sym_int4_g128"), writeback_stream=torch.cuda.Stream())
    with pytest.raises(ValueError):  # group 128 must divide the value dimension
        FormatStatePool(plan, 3, 64, get_format("sym_int4_g128"))
    assert isinstance(FormatStatePool(plan, 3, 64, get_format("fp32")), Fp32StatePool)
