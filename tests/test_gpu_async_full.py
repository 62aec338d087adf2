"""The asynchronous decode (readout + writeback) at the sizes the benchmark times.

The persistent readout and writeback kernels size their grid as resident CTAs
per SM x SMs, so only launches with more items than that make a CTA take a
second, third ... item: the carried (request, head) pair or the split of the
item index (a shift when the head count is a power of two, a division
otherwise), the slot ring and the swap of the two stage buffers.  These tests
launch 8,192 (GDN), 1,536 (24 heads: the division) and
16,384 (KDA, config 2) items per kernel and require, over three consecutive
steps:

* the async pool's page bytes equal the fused pool's (``sq_step``) exactly;
* the async readout equals the fused output bit for bit;
* the fused pages of sampled requests equal the oracle's ``page_encode`` of
  the fused kernel's own pre-quantization state (so the async bytes do too),
  and that state is within 1e-3 of the oracle's ``decode_step``; readouts
  within 2e-2 (bf16).

Reference semantics: stepquant/kernels/pool.py:200-297 (``step`` and
``_schedule_writeback``) and :299-316 (``_finish_update``).
"""
import numpy as np
import pytest
import torch

from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu


def _plan(arch, bits, seed):
    from stepquant_b200 import QuantizationPlan
    gen = torch.Generator().manual_seed(seed + 100)
    impact = torch.rand(bits.shape, generator=gen) + 0.25
    return QuantizationPlan(arch, bits.cuda(), impact.cuda()), O.Plan(arch, bits.numpy(), impact.numpy())


def _run(arch, plan, oplan, batch, heads, qk, seed, check):
    from stepquant_b200.kernels.pool import PackedStatePool
    kda = arch == "kda"
    gen = torch.Generator().manual_seed(seed)
    sync = PackedStatePool(plan, batch + 1, 128)
    asyn = PackedStatePool(plan, batch + 1, 128, writeback_stream=torch.cuda.Stream(), writeback_chunk=0)
    slots = torch.randperm(batch, generator=gen).cuda() + 1
    state = torch.randn(batch, heads, 128, 128, generator=gen).cuda() * 0.1
    sync.encode(state, slots)
    asyn.encode(state, slots)
    del state
    a_log = (torch.rand(heads, generator=gen) * np.log(16))
    dt_bias = torch.zeros(heads * 128 if kda else heads)
    kw = dict(normalize=True, scale=128 ** -0.5, a_log=a_log.cuda(), dt_bias=dt_bias.cuda())
    upd = torch.empty(batch, heads, 128, 128, device="cuda")
    s = slots.cpu().numpy()
    for step in range(3):
        q = torch.randn(batch, qk, 128, generator=gen).bfloat16()
        k = torch.randn(batch, qk, 128, generator=gen).bfloat16()
        v = torch.randn(batch, heads, 128, generator=gen).bfloat16()
        a = torch.randn(batch, heads, 128, generator=gen) if kda else torch.randn(batch, heads, generator=gen)
        b = torch.randn(batch, heads, generator=gen)
        before = sync.data[slots[check]].cpu().numpy()
        args = [t.cuda() for t in (q, k, v, a, b)]
        o_sync = sync.step(*args, slots, state_out=upd, **kw)
        o_async = asyn.step(*args, slots, **kw)
        asyn.wait()
        torch.cuda.synchronize()
        sync.check_status()
        asyn.check_status()
        assert torch.equal(o_sync, o_async), f"step {step}: async readout differs from the fused step"
        assert torch.equal(sync.data, asyn.data), f"step {step}: async page bytes differ from the fused step"
        if step == 0:
            pages = np.zeros((len(check) + 1, sync.page_bytes), np.uint8)
            pages[1:] = before
            o_out, _, o_upd = O.decode_step(pages, np.arange(1, len(check) + 1), oplan, 128, q[check].float().numpy(),
                                            k[check].float().numpy(), v[check].float().numpy(), a[check].numpy(),
                                            b[check].numpy(), normalize=True, scale=128 ** -0.5,
                                            a_log=a_log.numpy(), dt_bias=dt_bias.numpy())
            u = upd[check].cpu().numpy()
            assert np.abs(u - o_upd).max() <= 1e-3 * np.abs(o_upd).max()
            np.testing.assert_allclose(o_async[check].float().cpu().numpy(), o_out, atol=2e-2, rtol=0)
        u = upd[check].cpu().numpy()
        expected = O.page_encode(u, oplan, before)
        got = asyn.data.cpu().numpy()
        for j, i in enumerate(check):
            assert (got[s[i]] == expected[j]).all(), f"step {step}, request {i}: bytes differ from the oracle"


@pytest.mark.parametrize("pivot_heads", [0, 1])
def test_gdn_config1_async_full_size(pivot_heads):
    """B = 256, 32 value heads over 16 qk heads, widths {4, 6, 8} at 8/16/8
    (seed 1): 8,192 items per launch, the power-of-two item split.  With a
    fp16 pivot head the readout updates that head's values in place and the
    writeback leaves them."""
    from stepquant_b200 import synthetic as S
    gen = torch.Generator().manual_seed(1)
    widths = S.gdn_widths(32, gen, pivot_heads=pivot_heads)
    bits = widths[:, None].expand(32, 128).clone()
    plan, oplan = _plan("gdn", bits, 1)
    _run("gdn", plan, oplan, 256, 32, 16, 1, [0, 1, 77, 200, 255])


def test_gdn_non_power_of_two_heads_async_full_size():
    """24 value heads over 12 qk heads, B = 64: 1,536 items per launch, the
    item index split by division."""
    widths = torch.tensor([4, 6, 8, 6, 6, 4, 8, 6] * 3)
    bits = widths[:, None].expand(24, 128).clone()
    plan, oplan = _plan("gdn", bits, 2)
    _run("gdn", plan, oplan, 64, 24, 12, 2, [0, 31, 63])


def test_kda_config2_async_full_size():
    """KDA B = 512, 32 heads, per-row widths {2, 4, 6} at 30/50/20 with 2 %
    fp16 pivot rows: 16,384 items per launch."""
    from stepquant_b200 import synthetic as S
    gen = torch.Generator().manual_seed(2)
    bits = S.kda_widths(32, 128, gen)
    plan, oplan = _plan("kda", bits, 3)
    _run("kda", plan, oplan, 512, 32, 32, 3, [0, 5, 300, 511])


@pytest.mark.parametrize("per_sm, widths", [
    (7, [16, 6, 8, 4]),           # rank 0 of config 1 at 8 GPUs: three integer heads and the pivot head
    (4, [4, 6, 8, 6]),
    (8, [8, 4, 6, 6]),
    (10, [6, 4, 8, 6, 6, 4]),     # six heads: the item index split by division
])
def test_gdn_rank_sized_async(per_sm, widths):
    """Per-rank launches of a value-head-sharded config 1 (a few items per SM).
    When the busiest SM holds 4, 7, 8, 10 or 11 items the writeback runs four
    item groups per SM instead of three; the batch is chosen from this GPU's SM
    count so that it does, and the bytes must still equal the fused step's."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    heads = len(widths)
    batch = (per_sm * sms - heads + 1) // heads
    items = batch * heads
    assert -(-items // sms) == per_sm and items <= per_sm * sms
    bits = torch.tensor(widths)[:, None].expand(heads, 128).clone()
    plan, oplan = _plan("gdn", bits, 4 + per_sm)
    _run("gdn", plan, oplan, batch, heads, heads // 2, 4 + per_sm, [0, batch // 2, batch - 1])
