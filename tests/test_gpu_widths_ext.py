"""The 3- and 5-bit width extension on the device (``QuantizationPlan(...,
extended_widths=True)``; the reference admits 2, 4, 6, 8 and 16 only).

* device fit_state equals the reference's fit_state formula at those widths
  (golden vectors ``widths_ext.npz``, made by the unmodified reference with
  its width validation bypassed);
* ``pack`` / ``unpack`` at 3 and 5 bits equal the oracle's streams;
* encode, fused step and async step of GDN pages with 3- and 5-bit heads and
  of KDA pages with {3, 4, 6}-bit rows plus fp16 pivot rows (BASELINE config
  2's plan) write the oracle's page bytes for the kernels' own updated state;
  async bytes equal fused bytes.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def _cases():
    d = load_golden("widths_ext.npz")
    return sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_arch")})


@pytest.mark.parametrize("case", _cases())
def test_device_fit_state_at_extended_widths(case):
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.quantization import fit_state
    d = load_golden("widths_ext.npz")
    plan = QuantizationPlan(str(d[f"{case}_arch"]), torch.from_numpy(d[f"{case}_bits"].astype(np.int64)).cuda(),
                            torch.from_numpy(d[f"{case}_impact"]).cuda(), int(d[f"{case}_group"]), extended_widths=True)
    z, r, c, _, _ = fit_state(torch.from_numpy(d[f"{case}_x"]).cuda(), plan)
    assert (z.cpu().numpy() == d[f"{case}_z"]).all()
    assert (r.cpu().numpy().view(np.uint16) == d[f"{case}_r"].view(np.uint16)).all()
    assert (c.cpu().numpy().view(np.uint16) == d[f"{case}_c"].view(np.uint16)).all()


def test_pack_unpack_at_3_and_5_bits():
    from stepquant_b200.packing import pack, unpack
    gen = torch.Generator().manual_seed(60)
    for bits in (3, 5):
        for n in (1, 8, 37, 1000):
            codes = torch.randint(2 ** bits, (n,), generator=gen)
            data = pack(codes.cuda(), bits, extended=True)
            assert (data.cpu().numpy() == O.pack(codes.numpy(), bits, extended=True)).all()
            assert torch.equal(unpack(data, bits, n, extended=True).cpu(), codes.to(torch.int16))
        with pytest.raises(ValueError):
            pack(codes.cuda(), bits)


def _plans(arch, seed):
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200 import synthetic as S
    gen = torch.Generator().manual_seed(seed)
    if arch == "gdn":
        bits = torch.tensor([3, 5, 4, 6, 5, 3, 16, 8])[:, None].expand(8, 128).clone()
    else:
        bits = S.kda_widths(8, 128, gen, choices=(3, 4, 6), probs=(0.3, 0.5, 0.2), pivot_fraction=0.02)
    impact = torch.rand(bits.shape, generator=gen) + 0.25
    plan = QuantizationPlan(arch, bits.cuda(), impact.cuda(), extended_widths=True)
    return plan, O.Plan(arch, bits.numpy(), impact.numpy(), extended_widths=True)


@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_extended_pages_encode_step_and_async(arch):
    from stepquant_b200.kernels.pool import PackedStatePool
    plan, oplan = _plans(arch, 61 if arch == "gdn" else 62)
    heads, batch = 8, 24
    gen = torch.Generator().manual_seed(63)
    sync = PackedStatePool(plan, batch + 1, 128)
    asyn = PackedStatePool(plan, batch + 1, 128, writeback_stream=torch.cuda.Stream())
    slots = torch.randperm(batch, generator=gen).cuda() + 1
    state = torch.randn(batch, heads, 128, 128, generator=gen) * 0.1
    before = sync.data.cpu().numpy()
    sync.encode(state.cuda(), slots)
    asyn.encode(state.cuda(), slots)
    s = slots.cpu().numpy()
    expected = O.page_encode(state.numpy(), oplan, before[s])
    assert (sync.data.cpu().numpy()[s] == expected).all(), "encode bytes"
    kda = arch == "kda"
    qk = heads if kda else heads // 2
    a_log = torch.rand(heads, generator=gen)
    dt_bias = torch.zeros(heads * 128 if kda else heads)
    kw = dict(normalize=True, scale=128 ** -0.5, a_log=a_log.cuda(), dt_bias=dt_bias.cuda())
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    for step in range(2):
        q = torch.randn(batch, qk, 128, generator=gen).bfloat16()
        k = torch.randn(batch, qk, 128, generator=gen).bfloat16()
        v = torch.randn(batch, heads, 128, generator=gen).bfloat16()
        a = torch.randn(batch, heads, 128, generator=gen) if kda else torch.randn(batch, heads, generator=gen)
        b = torch.randn(batch, heads, generator=gen)
        prior = sync.data.cpu().numpy()
        args = [t.cuda() for t in (q, k, v, a, b)]
        o1 = sync.step(*args, slots, state_out=upd, **kw)
        o2 = asyn.step(*args, slots, **kw)
        asyn.wait()
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        assert torch.equal(sync.data, asyn.data), f"step {step}: async bytes differ from fused"
        pick = [0, 5, 23]
        o_out, _, o_upd = O.decode_step(prior, s[pick], oplan, 128, q[pick].float().numpy(), k[pick].float().numpy(),
                                        v[pick].float().numpy(), a[pick].numpy(), b[pick].numpy(), normalize=True,
                                        scale=128 ** -0.5, a_log=a_log.numpy(), dt_bias=dt_bias.numpy())
        u = upd.cpu().numpy()[pick]
        assert np.abs(u - o_upd).max() <= 1e-3 * np.abs(o_upd).max()
        np.testing.assert_allclose(o1.float().cpu().numpy()[pick], o_out, atol=2e-2, rtol=0)
        expected = O.page_encode(u, oplan, prior[s[pick]])
        got = sync.data.cpu().numpy()
        for j, i in enumerate(pick):
            assert (got[s[i]] == expected[j]).all(), f"step {step}, request {i}: bytes differ from the oracle"
