"""Register-resident K = V = 128 GDN kernels (csrc/sq_fast.cu) against the oracle and the tile kernel.

* the fp16-divisor division equals IEEE a / b (exhaustive over the fp16
  divisors for a sample of dividends, plus dividends next to rounding midpoints);
* full-size steps (batch 256, 32 heads of widths 4/6/8)
  repack bit-exactly what the oracle's fit_state gives for the kernel's own
  pre-quantization state, readout within atol 5e-5 / rtol 1e-4 (fp32 out) and
  2e-2 (bf16 out);
* plans mixing fast heads with 2-bit and fp16 pivot heads (tile kernel) work;
* async (readout + writeback) bytes == fused bytes at full size; graph replay.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def test_fp16_divisor_division_is_ieee():
    from stepquant_b200 import _native as N
    divisors = torch.arange(1, 0x7C00, dtype=torch.int32)  # every positive finite fp16
    divisors = divisors[(divisors & 0x3FF) != 0x3FF]  # keep the sweep size round; spot values below
    gen = torch.Generator().manual_seed(0)
    for scale in (1e-3, 1.0, 37.0, 1e4):
        a = (torch.randn(divisors.numel(), generator=gen) * scale).float()
        b = divisors.to(torch.int16).view(torch.int16)
        out = torch.empty_like(a, device="cuda")
        a_d, b_d = a.cuda(), b.cuda()
        N.check(N.lib().sq_selftest_fp16_division(N.ptr(a_d), N.ptr(b_d), N.ptr(out), a.numel(), N.stream_handle()))
        ieee = a_d / b_d.view(torch.float16).float()
        torch.cuda.synchronize()
        normal = ieee.abs() >= 2.0 ** -100
        assert torch.equal(out[normal], ieee[normal])
    # Dividends one ulp around b * (m + 1/2) (quotients next to rounding midpoints).
    b16 = torch.tensor([0.1, 0.3, 1.7, 3.0, 0.0056, 129.5, 2.0 ** -20], dtype=torch.float16)
    m = torch.arange(1, 2000, dtype=torch.float64)
    rows = []
    for bv in b16.tolist():
        mid = torch.tensor(bv, dtype=torch.float64) * (m + 0.5)
        base = mid.float()
        for d in (-2, -1, 0, 1, 2):
            rows.append((torch.nextafter(base, torch.tensor(np.inf if d > 0 else -np.inf)) if d else base,
                         torch.full_like(base, bv)))
    a = torch.cat([r[0] for r in rows]).cuda()
    b = torch.cat([r[1] for r in rows]).half().view(torch.int16).cuda()
    out = torch.empty_like(a)
    N.check(N.lib().sq_selftest_fp16_division(N.ptr(a), N.ptr(b), N.ptr(out), a.numel(), N.stream_handle()))
    assert torch.equal(out, a / b.view(torch.float16).float())


def _gdn_plan(widths, seed=0):
    from stepquant_b200 import QuantizationPlan
    gen = torch.Generator().manual_seed(seed)
    heads = len(widths)
    bits = torch.tensor(widths)[:, None].expand(heads, 128).clone()
    impact = torch.rand(heads, 128, generator=gen) + 0.25
    return QuantizationPlan("gdn", bits.cuda(), impact.cuda()), O.Plan("gdn", bits.numpy(), impact.numpy())


def _inputs(batch, heads, qk_heads, gen, dtype):
    q = torch.randn(batch, qk_heads, 128, generator=gen).to(dtype)
    k = torch.randn(batch, qk_heads, 128, generator=gen).to(dtype)
    v = torch.randn(batch, heads, 128, generator=gen).to(dtype)
    a = torch.randn(batch, heads, generator=gen)
    b = torch.randn(batch, heads, generator=gen)
    return q, k, v, a, b


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_config1_step_bytes_exact_and_readout(dtype):
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(1)
    widths = [4] * 8 + [6] * 16 + [8] * 8
    widths = [widths[i] for i in torch.randperm(32, generator=gen).tolist()]
    plan, oplan = _gdn_plan(widths, 1)
    batch, heads, qk = 256, 32, 16
    pool = PackedStatePool(plan, batch + 1, 128)
    slots = torch.arange(1, batch + 1, device="cuda")
    slots[17] = 0
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.1
    pool.encode(state, slots)
    a_log = torch.rand(heads) * np.log(16)
    dt_bias = torch.zeros(heads)
    q, k, v, a, b = _inputs(batch, heads, qk, gen, dtype)
    before = pool.data.cpu().numpy()
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    out = pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, normalize=True, scale=128 ** -0.5,
                    a_log=a_log.cuda(), dt_bias=dt_bias.cuda(), state_out=upd)
    pool.check_status()
    pages = pool.data.cpu().numpy()
    s = slots.cpu().numpy()
    check = [0, 1, 16, 100, 255]  # requests compared with the oracle (the full batch is too slow on CPU)
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
    assert out[17].count_nonzero() == 0 and (pages[0] == before[0]).all()
    # Every request: the fast kernel's bytes requantize its own state exactly
    # (compared through the tile kernel's encode of that state).
    pool2 = PackedStatePool(plan, batch + 1, 128)
    active = slots > 0
    pool2.encode(upd[active], slots[active])
    assert torch.equal(pool2.data[slots[active]], pool.data[slots[active]])


def test_mixed_fast_and_tile_heads_async_equals_fused():
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(5)
    plan, oplan = _gdn_plan([6, 16, 4, 2, 8, 6], 5)
    batch, heads, qk = 40, 6, 3
    sync = PackedStatePool(plan, batch + 2, 128)
    asyn = PackedStatePool(plan, batch + 2, 128, writeback_stream=torch.cuda.Stream())
    slots = torch.randperm(batch + 1, generator=gen)[:batch].cuda() + 1
    slots[3] = 0
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.2
    sync.encode(state, slots)
    asyn.encode(state, slots)
    a_log, dt_bias = torch.rand(heads).cuda(), torch.zeros(heads).cuda()
    for step in range(3):
        q, k, v, a, b = (t.cuda() for t in _inputs(batch, heads, qk, gen, torch.bfloat16))
        before = sync.data.cpu().numpy()
        upd = torch.empty(batch, heads, 128, 128, device="cuda")
        o1 = sync.step(q, k, v, a, b, slots, normalize=True, scale=128 ** -0.5, a_log=a_log, dt_bias=dt_bias,
                       state_out=upd)
        o2 = asyn.step(q, k, v, a, b, slots, normalize=True, scale=128 ** -0.5, a_log=a_log, dt_bias=dt_bias)
        asyn.wait()
        torch.cuda.synchronize()
        assert torch.equal(o1, o2)
        assert torch.equal(sync.data, asyn.data), f"step {step}"
        s = slots.cpu().numpy()
        pick = [0, 1, 2, 7]
        expected = O.page_encode(upd.cpu().numpy()[pick], oplan, before[s[pick]])
        got = sync.data.cpu().numpy()
        for j, i in enumerate(pick):
            assert (got[s[i]] == expected[j]).all()


def test_fast_path_graph_capture():
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.writeback import WritebackGraph, attention_window, defer_writeback
    gen = torch.Generator().manual_seed(9)
    plan, _ = _gdn_plan([4, 6, 8, 6], 9)
    batch, heads = 64, 4
    stream = torch.cuda.Stream()
    pools = [PackedStatePool(plan, batch + 1, 128, writeback_stream=stream, writeback_chunk=16) for _ in range(2)]
    refs = [PackedStatePool(plan, batch + 1, 128) for _ in range(2)]
    slots = torch.arange(batch, 0, -1, device="cuda")
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.1
    for p in pools + refs:
        p.encode(state, slots)
    q, k, v, a, b = (t.cuda() for t in _inputs(batch, heads, heads, gen, torch.bfloat16))
    kw = dict(normalize=True, scale=128 ** -0.5, a_log=torch.rand(heads).cuda(), dt_bias=torch.zeros(heads).cuda())
    for p in pools:
        p.step(q, k, v, a, b, slots, **kw)
        p.wait()
    for p in refs:
        p.step(q, k, v, a, b, slots, **kw)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        with defer_writeback(pools, attention_windows=True) as tasks:
            outs = []
            for p in pools:
                attention_window()
                outs.append(p.step(q, k, v, a, b, slots, **kw))
                attention_window()
    wg = WritebackGraph(graph, tasks)
    for _ in range(3):
        wg.replay()
        expected = [r.step(q, k, v, a, b, slots, **kw) for r in refs]
        for p in pools:
            p.wait()
        torch.cuda.synchronize()
        for o, e in zip(outs, expected):
            assert torch.equal(o, e)
        for p, r in zip(pools, refs):
            assert torch.equal(p.data, r.data)


def test_joined_capture_of_chained_layers():
    """Three layers captured in one graph with joined writeback (the decode
    stack of the benchmark's config 4): each layer's v is fed by the previous
    layer's readout; replays equal eager fused steps, outputs and bytes."""
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.writeback import WritebackGraph, defer_writeback
    gen = torch.Generator().manual_seed(10)
    plan, _ = _gdn_plan([6, 8, 4, 6], 10)
    batch, heads, layers = 96, 4, 3
    stream = torch.cuda.Stream()
    pools = [PackedStatePool(plan, batch + 1, 128, writeback_stream=stream, writeback_chunk=32) for _ in range(layers)]
    refs = [PackedStatePool(plan, batch + 1, 128) for _ in range(layers)]
    slots = torch.randperm(batch, generator=gen).cuda() + 1
    state = torch.randn(batch, heads, 128, 128, device="cuda") * 0.1
    for p in pools + refs:
        p.encode(state, slots)
    q, k, v, a, b = (t.cuda() for t in _inputs(batch, heads, heads, gen, torch.bfloat16))
    kw = dict(normalize=True, scale=128 ** -0.5, a_log=torch.rand(heads).cuda(), dt_bias=torch.zeros(heads).cuda())
    v_in = v.clone()

    def forward(stack):
        x, outs = v_in, []
        for p in stack:
            out = p.step(q, k, x, a, b, slots, **kw)
            outs.append(out)
            x = (x.float() + out.float()).bfloat16()
        return outs

    forward(pools)  # eager warm-up step on both sets
    forward(refs)
    for p in pools:
        p.wait()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        with defer_writeback(pools, joined=True) as tasks:
            outs = forward(pools)
    wg = WritebackGraph(graph, tasks, joined=True)
    assert wg.background is None
    for step in range(3):
        v_in.copy_(torch.randn(v.shape, generator=gen).bfloat16())
        wg.replay()
        expected = forward(refs)
        for p in pools:
            p.wait()
        torch.cuda.synchronize()
        for o, e in zip(outs, expected):
            assert torch.equal(o, e), f"step {step}"
        for p, r in zip(pools, refs):
            assert torch.equal(p.data, r.data), f"step {step}"


def test_ieee_path_rows_beyond_2_96():
    """Rows whose |x| sum exceeds 2^96 switch a tile to IEEE divisions (the
    kernels' SLOW path, reached by the encode of such a state): the pages equal
    the oracle's.  The decoded state is bounded by the saturated fp16 scales
    (65504^2 * qmax), so the following step runs the ordinary path on tiles
    whose r and c saturate; its bytes equal the oracle's too."""
    from stepquant_b200.kernels.pool import PackedStatePool
    gen = torch.Generator().manual_seed(12)
    plan, oplan = _gdn_plan([4, 6, 8, 6], 12)
    batch, heads = 6, 4
    pool = PackedStatePool(plan, batch + 1, 128)
    slots = torch.arange(1, batch + 1, device="cuda")
    state = torch.randn(batch, heads, 128, 128, generator=gen) * 0.1
    state[1, :, 5] *= 1e28   # |x| row sums near 1e29 > 2^96 in every head of request 1
    state[3, 2, 100] *= 3e27
    before = pool.data.cpu().numpy()
    pool.encode(state.cuda(), slots)
    expected = O.page_encode(state.numpy(), oplan, before[1:])
    got = pool.data.cpu().numpy()
    for i in range(batch):
        assert (got[i + 1] == expected[i]).all(), f"encode, request {i}"
    q, k, v, a, b = _inputs(batch, heads, heads, gen, torch.float32)
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    before = pool.data.cpu().numpy()
    pool.step(q.cuda(), k.cuda(), v.cuda(), a.cuda(), b.cuda(), slots, normalize=True, scale=128 ** -0.5,
              a_log=torch.rand(heads).cuda(), dt_bias=torch.zeros(heads).cuda(), state_out=upd)
    pool.check_status()
    u = upd.cpu().numpy()
    assert np.isfinite(u).all() and np.abs(u).max() > 1e9
    expected = O.page_encode(u, oplan, before[1:])
    got = pool.data.cpu().numpy()
    for i in range(batch):
        assert (got[i + 1] == expected[i]).all(), f"step, request {i}"
