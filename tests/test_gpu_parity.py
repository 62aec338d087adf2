"""CUDA path vs the CPU oracle (and the reference's golden vectors), through the C ABI.

Criteria (written per test):
* page bytes, integer levels and fp16 scales: bit-exact -- given the same fp32
  pre-quantization state, the device quantizer must produce the reference
  quantizer's bytes;
* the recurrent update before requantization: max relative error 1e-3 of the
  state scale (north star), and the reference tests' atol 5e-5 / rtol 1e-4 on
  fp32 outputs, atol 2e-2 on bf16 outputs;
* asynchronous (readout + writeback) and synchronous (fused) steps write the
  same bytes.
"""
import numpy as np
import pytest
import torch

from conftest import golden_fit_cases, load_golden
from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def _plans(d, device="cuda"):
    from stepquant_b200 import QuantizationPlan
    bits = torch.from_numpy(d["bits"].astype(np.int64))
    impact = torch.from_numpy(d["impact"])
    arch = str(d["architecture"])
    group = int(d["group"])
    return (QuantizationPlan(arch, bits.to(device), impact.to(device), group),
            O.Plan(arch, bits.numpy(), impact.numpy(), group))


def _pool(plan, slots, values, stream=None):
    from stepquant_b200.kernels.pool import PackedStatePool
    return PackedStatePool(plan, slots, values, writeback_stream=stream)


@pytest.mark.parametrize("case", golden_fit_cases())
def test_fit_state_bit_exact_with_reference(case):
    from stepquant_b200 import fit_state
    d = load_golden(f"fit_{case}.npz")
    plan, _ = _plans(d)
    z, r, c, r2, recon = fit_state(torch.from_numpy(d["x"]).cuda(), plan)
    torch.cuda.synchronize()
    assert (z.cpu().numpy() == d["z"]).all()
    assert (r.cpu().numpy().view(np.uint16) == d["r"].view(np.uint16)).all()
    assert (c.cpu().numpy().view(np.uint16) == d["c"].view(np.uint16)).all()
    if "r2" in d:
        assert (r2.cpu().numpy().view(np.uint16) == d["r2"].view(np.uint16)).all()
    oracle_recon = O.fit_state(d["x"], _plans(d)[1])[-1]
    assert (recon.cpu().numpy() == oracle_recon).all()


@pytest.mark.parametrize("case", golden_fit_cases())
def test_encode_decode_pages_bit_exact(case):
    d = load_golden(f"fit_{case}.npz")
    plan, oplan = _plans(d)
    batch, values = d["x"].shape[0], d["x"].shape[-1]
    pool = _pool(plan, batch + 2, values)
    slots = torch.arange(batch, 0, -1, device="cuda")
    pool.encode(torch.from_numpy(d["x"]).cuda(), slots)
    expected = O.page_encode(d["x"], oplan)
    got = pool.data.cpu().numpy()
    for i, s in enumerate(slots.tolist()):
        assert (got[s] == expected[i]).all(), f"page bytes differ for request {i}"
    assert (got[0] == 0).all() and (got[batch + 1] == 0).all()
    decoded = pool.decode(slots).cpu().numpy()
    assert (decoded == O.fit_state(d["x"], oplan)[-1]).all()
    # Padded slots decode to zeros.
    assert pool.decode(torch.tensor([0, -3], device="cuda")).count_nonzero() == 0


def _gates(arch, batch, heads, keys, gen, raw):
    if raw:
        a = torch.randn(batch, heads, keys, generator=gen) if arch == "kda" else torch.randn(batch, heads, generator=gen)
        b = torch.randn(batch, heads, generator=gen)
        a_log = torch.rand(heads, generator=gen) * np.log(16)
        dt_bias = torch.randn(heads * keys if arch == "kda" else heads, generator=gen) * 0.1
        return a, b, a_log, dt_bias
    g = -torch.rand(batch, heads, keys, generator=gen) if arch == "kda" else -torch.rand(batch, heads, generator=gen)
    return g, torch.rand(batch, heads, generator=gen), None, None


@pytest.mark.parametrize("case", ["gdn_mixed_k32", "kda_mixed_k32", "gdn_k128", "kda_k128", "gdn_k4_v8",
                                  "kda_k4_v4_half", "kda_k64_v8", "gdn_k128_v16"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("raw", [False, True])
def test_step_against_oracle(case, dtype, raw):
    d = load_golden(f"fit_{case}.npz")
    plan, oplan = _plans(d)
    x = d["x"]
    batch, heads, keys, values = x.shape
    batch_total = batch + 1
    pool = _pool(plan, batch + 3, values)
    slots = torch.tensor(list(range(batch, 0, -1)) + [0], device="cuda")
    pool.encode(torch.from_numpy(x).cuda(), slots[:-1])
    gen = torch.Generator().manual_seed(7)
    qk_heads = max(1, heads // 2) if heads % 2 == 0 else heads
    q = torch.randn(batch_total, qk_heads, keys, generator=gen)
    k = torch.randn(batch_total, qk_heads, keys, generator=gen)
    v = torch.randn(batch_total, heads, values, generator=gen)
    g, beta, a_log, dt_bias = _gates(oplan.architecture, batch_total, heads, keys, gen, raw)
    before = pool.data.cpu().numpy()
    state_out = torch.empty(batch_total, heads, keys, values, device="cuda")
    prep = dict(normalize=True, scale=keys ** -0.5)
    if raw:
        prep.update(a_log=a_log.cuda(), dt_bias=dt_bias.cuda())
    out = pool.step(q.to(dtype).cuda(), k.to(dtype).cuda(), v.to(dtype).cuda(), g.cuda(), beta.cuda(), slots,
                    state_out=state_out, **prep)
    pool.check_status()
    oprep = dict(normalize=True, scale=keys ** -0.5)
    if raw:
        oprep.update(a_log=a_log.numpy(), dt_bias=dt_bias.numpy())
    qn, kn, vn = (t.to(dtype).float().numpy() for t in (q, k, v))
    o_out, o_pages, o_updated = O.decode_step(before, slots.cpu().numpy(), oplan, values, qn, kn, vn,
                                              g.numpy(), beta.numpy(), **oprep)
    upd = state_out.cpu().numpy()
    scale = np.abs(o_updated).max() + 1e-30
    assert np.abs(upd[:-1] - o_updated[:-1]).max() <= 1e-3 * scale
    got = out.float().cpu().numpy()
    if dtype == torch.float32:
        np.testing.assert_allclose(got[:-1], o_out[:-1], atol=5e-5, rtol=1e-4)
    else:
        np.testing.assert_allclose(got[:-1], o_out[:-1], atol=2e-2, rtol=0)
    assert (got[-1] == 0).all()
    # Bit-exact requantization of the kernel's own pre-quantization state.
    pages = pool.data.cpu().numpy()
    expected = O.page_encode(upd[:-1], oplan, before[slots[:-1].cpu().numpy()])
    for i, s in enumerate(slots[:-1].tolist()):
        assert (pages[s] == expected[i]).all(), f"request {i}: packed bytes differ"
    assert (pages[0] == 0).all()


@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_async_writeback_matches_fused_bytes(arch):
    from stepquant_b200 import QuantizationPlan
    torch.manual_seed(3)
    heads, keys, values, batch = 5, 128, 128, 9
    if arch == "gdn":
        bits = torch.tensor([4, 6, 8, 16, 2])[:, None].expand(heads, keys).clone()
    else:
        bits = torch.tensor([2, 4, 6, 8])[torch.randint(0, 4, (heads, keys))]
        bits[torch.rand(heads, keys) < 0.05] = 16
    plan = QuantizationPlan(arch, bits.cuda(), (torch.rand(heads, keys) + 0.3).cuda())
    sync = _pool(plan, batch + 1, values)
    asyn = _pool(plan, batch + 1, values, torch.cuda.Stream())
    slots = torch.arange(1, batch + 1, device="cuda")
    slots[3] = 0
    state = torch.randn(batch, heads, keys, values, device="cuda") * 0.1
    sync.encode(state, slots)
    asyn.encode(state, slots)
    for step in range(3):
        q = torch.randn(batch, heads, keys, device="cuda", dtype=torch.bfloat16)
        k = torch.randn_like(q)
        v = torch.randn(batch, heads, values, device="cuda", dtype=torch.bfloat16)
        g = torch.randn(batch, heads, keys, device="cuda") if arch == "kda" else torch.randn(batch, heads, device="cuda")
        b = torch.randn(batch, heads, device="cuda")
        kw = dict(normalize=True, scale=keys ** -0.5, a_log=torch.rand(heads, device="cuda"),
                  dt_bias=torch.zeros(heads * keys if arch == "kda" else heads, device="cuda"))
        o1 = sync.step(q, k, v, g, b, slots, **kw)
        o2 = asyn.step(q, k, v, g, b, slots, **kw)
        asyn.wait()
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        assert torch.equal(sync.data, asyn.data), f"step {step}: async bytes differ from fused bytes"
        # In-place reuse of scheduler metadata while the side stream runs (test_fused_cuda.py:99-117).
        slots.fill_(7)
        slots.copy_(torch.tensor([1, 2, 3, 0, 5, 6, 7, 8, 9], device="cuda"))


def test_slot_out_of_range_is_flagged_and_skipped():
    from stepquant_b200 import QuantizationPlan
    plan = QuantizationPlan("gdn", torch.full((2, 32), 6, device="cuda"), torch.ones(2, 32, device="cuda"))
    pool = _pool(plan, 4, 32)
    q = torch.randn(2, 2, 32, device="cuda")
    out = pool.step(q, q, torch.randn(2, 2, 32, device="cuda"), -torch.rand(2, 2, device="cuda"),
                    torch.rand(2, 2, device="cuda"), torch.tensor([2, 9], device="cuda"))
    torch.cuda.synchronize()
    assert out[1].count_nonzero() == 0
    with pytest.raises(IndexError):
        pool.check_status()
    pool.check_status()  # the flag is cleared once reported


def test_pack_unpack_against_reference_vectors():
    from stepquant_b200.packing import pack, unpack
    d = load_golden("pack.npz")
    for bits in (2, 4, 6, 8):
        for n in (0, 1, 7, 128, 513):
            codes = torch.from_numpy(d[f"codes_{bits}_{n}"]).cuda()
            packed = pack(codes, bits)
            assert (packed.cpu().numpy() == d[f"packed_{bits}_{n}"]).all()
            assert torch.equal(unpack(packed, bits, n), codes)


@pytest.mark.parametrize("case", ["gdn_mixed_k32_g8", "kda_mixed_k32", "gdn_k128"])
def test_state_codec_streams_match_reference(case):
    from stepquant_b200 import StateCodec
    d = load_golden(f"fit_{case}.npz")
    plan, _ = _plans(d)
    codec = StateCodec(plan)
    packed = codec.encode(torch.from_numpy(d["x"]).cuda())
    for b in (2, 4, 6, 8):
        assert (packed.codes[b].cpu().numpy() == d[f"codes{b}"]).all()
    assert (packed.rows.cpu().numpy().view(np.uint16) == d["rows"].view(np.uint16)).all()
    assert (packed.pivots.cpu().numpy().view(np.uint16) == d["pivots"].view(np.uint16)).all()
    recon = O.fit_state(d["x"], _plans(d)[1])[-1]
    np.testing.assert_allclose(codec.decode(packed).cpu().numpy(), recon, atol=1e-6, rtol=1e-6)


@pytest.mark.parametrize("asynchronous", [False, True])
def test_cuda_graph_replay_matches_eager(asynchronous):
    from stepquant_b200 import QuantizationPlan
    torch.manual_seed(8)
    heads, qk, keys, values, batch = 4, 2, 32, 32, 16
    plan = QuantizationPlan("gdn", torch.tensor([4, 6, 8, 16])[:, None].expand(heads, keys).clone().cuda(),
                            torch.rand(heads, keys, device="cuda") + 0.5)
    stream = torch.cuda.Stream() if asynchronous else None
    pool = _pool(plan, batch + 1, values, stream)
    ref = _pool(plan, batch + 1, values, stream and torch.cuda.Stream())
    slots = torch.arange(batch - 1, -1, -1, device="cuda")
    mixed = torch.randn(batch, 2 * qk * keys + heads * values, device="cuda", dtype=torch.bfloat16)
    q, k, v = mixed.split([qk * keys, qk * keys, heads * values], -1)
    a = torch.randn(batch, heads, device="cuda")
    b = torch.randn(batch, heads, device="cuda")
    kw = dict(normalize=True, scale=keys ** -0.5, a_log=torch.randn(heads, device="cuda"),
              dt_bias=torch.randn(heads, device="cuda"))

    def call(p):
        return p.step(q, k, v, a, b, slots, **kw)

    call(pool)
    pool.wait()
    call(ref)
    ref.wait()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = call(pool)
        pool.wait()
    for _ in range(3):
        graph.replay()
        expected = call(ref)
        ref.wait()
        torch.cuda.synchronize()
        assert torch.equal(out, expected)
        assert torch.equal(pool.data, ref.data)
        assert out[-1].count_nonzero() == 0 and pool.data[0].count_nonzero() == 0


def test_fp32_pool_step_matches_oracle():
    from stepquant_b200 import _native as N
    import ctypes
    torch.manual_seed(4)
    for kda in (0, 1):
        heads, keys, values, batch = 3, 128, 64, 5
        state = torch.randn(batch + 1, heads, keys, values, device="cuda")
        before = state.clone()
        slots = torch.tensor([1, 2, 0, 4, 5], device="cuda")
        q = torch.randn(batch, heads, keys, device="cuda")
        k = torch.nn.functional.normalize(torch.randn_like(q), dim=-1)
        v = torch.randn(batch, heads, values, device="cuda")
        g = -torch.rand(batch, heads, keys, device="cuda") if kda else -torch.rand(batch, heads, device="cuda")
        beta = torch.rand(batch, heads, device="cuda")
        out = torch.empty(batch, heads, values, device="cuda")
        args = N.SqStepArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), k.stride(0), v.stride(0), heads,
                            N.SQ_F32, g.data_ptr(), beta.data_ptr(), N.SQ_F32, 0, None, None, 1.0, 0, out.data_ptr())
        N.check(N.lib().sq_fp32_step(N.ptr(state), batch + 1, heads, keys, values, kda, N.ptr(slots), batch,
                                     ctypes.byref(args), None, N.stream_handle()))
        torch.cuda.synchronize()
        s = slots.cpu().numpy()
        o_out, o_upd = O.delta_step(before.cpu().numpy()[np.maximum(s, 0)], q.cpu().numpy(), k.cpu().numpy(),
                                    v.cpu().numpy(), g.cpu().numpy(), beta.cpu().numpy())
        active = s > 0
        np.testing.assert_allclose(out.cpu().numpy()[active], o_out[active], atol=5e-5, rtol=1e-4)
        np.testing.assert_allclose(state.cpu().numpy()[s[active]], o_upd[active], atol=5e-5, rtol=1e-4)
        assert out[2].count_nonzero() == 0
