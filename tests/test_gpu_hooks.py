"""The SGLang hook functions and the FP32 baseline pool on the device."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _plan(heads=4, keys=128, arch="gdn"):
    from stepquant_b200 import QuantizationPlan
    bits = torch.tensor([4, 6, 8, 6])[:heads, None].expand(heads, keys).clone()
    return QuantizationPlan(arch, bits.cuda(), (torch.rand(heads, keys) + 0.5).cuda())


def test_packed_decode_hook_equals_pool_step():
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.sglang import runtime
    torch.manual_seed(0)
    heads, qk, keys, batch = 4, 2, 128, 6
    plan = _plan(heads, keys)
    pools = [PackedStatePool(plan, batch + 1, keys) for _ in range(2)]
    slots = torch.arange(1, batch + 1, device="cuda")
    state = torch.randn(batch, heads, keys, keys, device="cuda") * 0.1
    for p in pools:
        p.encode(state, slots)
    mixed = torch.randn(batch, 2 * qk * keys + heads * keys, device="cuda", dtype=torch.bfloat16)
    a = torch.randn(batch, heads, device="cuda")
    b = torch.randn(batch, heads, device="cuda")
    a_log, dt_bias = torch.rand(heads, device="cuda"), torch.zeros(heads, device="cuda")
    out = runtime.kernel_packed_decode(None, None, mixed, a, b, A_log=a_log, dt_bias=dt_bias, scale=keys ** -0.5,
                                       ssm_states=pools[0], cache_indices=slots, num_v_heads=heads, head_v_dim=keys)
    q, k, v = mixed.split([qk * keys, qk * keys, heads * keys], -1)
    ref = pools[1].step(q, k, v, a, b, slots, normalize=True, scale=keys ** -0.5, a_log=a_log, dt_bias=dt_bias)
    assert out.shape == (1, batch, heads, keys)
    assert torch.equal(out[0], ref) and torch.equal(pools[0].data, pools[1].data)


def test_extend_hook_round_trips_pages_through_native_kernel():
    """Pools the native passes do not cover (here KDA with K = V = 64): the
    original chunk kernel runs on the decoded V-first state."""
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.sglang import runtime
    torch.manual_seed(1)
    heads, keys, batch = 4, 64, 3
    plan = _plan(heads, keys, "kda")
    pool = PackedStatePool(plan, batch + 1, keys)
    slots = torch.tensor([2, 3, 1], device="cuda")
    seen = {}

    def native(self, q, k, v, g, beta, *, ssm_states, cache_indices, query_start_loc):
        seen["state"] = ssm_states.clone()          # V-first dense state of the active slots
        ssm_states.mul_(0.5)                        # the native chunk kernel updates it in place
        return "out"

    state = torch.randn(batch, heads, keys, keys, device="cuda") * 0.1
    pool.encode(state, slots)
    before = pool.decode(slots)
    assert runtime.kernel_extend(native, None, 0, 0, 0, 0, 0, ssm_states=pool, cache_indices=slots,
                                 query_start_loc=None) == "out"
    assert torch.equal(seen["state"], before.transpose(-1, -2))
    expected = PackedStatePool(plan, batch + 1, keys)
    expected.encode(before * 0.5, slots)
    assert torch.equal(pool.data, expected.data)


def test_extend_hook_runs_native_gdn_prefill():
    """GDN pools: the hook is PackedStatePool.extend (decode, chunk pass, encode)."""
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.sglang import runtime
    torch.manual_seed(3)
    heads, qk, keys = 4, 2, 128
    plan = _plan(heads, keys)
    pools = [PackedStatePool(plan, 5, keys) for _ in range(2)]
    slots = torch.tensor([3, 1], device="cuda")
    cu = torch.tensor([0, 70, 90], device="cuda", dtype=torch.int32)
    q, k = (torch.randn(1, 90, qk, keys, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    v = torch.randn(1, 90, heads, keys, device="cuda", dtype=torch.bfloat16)
    g = -torch.rand(1, 90, heads, device="cuda")
    beta = torch.rand(1, 90, heads, device="cuda")

    def original(*args, **kwargs):
        raise AssertionError("GDN prefill must not call the original kernel")

    out = runtime.kernel_extend(original, None, q, k, v, g, beta, ssm_states=pools[0], cache_indices=slots,
                                query_start_loc=cu)
    ref = pools[1].extend(q, k, v, g, beta, slots, cu)
    assert out.shape == (1, 90, heads, keys)
    assert torch.equal(out, ref) and torch.equal(pools[0].data, pools[1].data)


def test_extend_hook_runs_native_kda_prefill():
    """KDA pools with K = V = 128: the hook is PackedStatePool.extend (decode,
    the recurrent KDA pass with g per key channel, encode)."""
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.sglang import runtime
    torch.manual_seed(4)
    heads, keys = 4, 128
    plan = _plan(heads, keys, "kda")
    pools = [PackedStatePool(plan, 5, keys) for _ in range(2)]
    slots = torch.tensor([2, 4], device="cuda")
    cu = torch.tensor([0, 33, 80], device="cuda", dtype=torch.int32)
    q, k = (torch.randn(1, 80, heads, keys, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    v = torch.randn(1, 80, heads, keys, device="cuda", dtype=torch.bfloat16)
    g = -torch.rand(1, 80, heads, keys, device="cuda")
    beta = torch.rand(1, 80, heads, device="cuda")

    def original(*args, **kwargs):
        raise AssertionError("KDA prefill at K = V = 128 must not call the original kernel")

    out = runtime.kernel_extend(original, None, q, k, v, g, beta, ssm_states=pools[0], cache_indices=slots,
                                query_start_loc=cu)
    ref = pools[1].extend(q, k, v, g, beta, slots, cu)
    assert out.shape == (1, 80, heads, keys)
    assert torch.equal(out, ref) and torch.equal(pools[0].data, pools[1].data)


@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_fp32_pool_matches_packed_readout_semantics(arch):
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.formats import get_format
    from stepquant_b200.kernels.format_pool import Fp32StatePool
    from oracle import stepquant_oracle as O
    torch.manual_seed(2)
    heads, keys, batch = 3, 64, 4
    plan = QuantizationPlan(arch, torch.full((heads, keys), 6).cuda(), torch.ones(heads, keys).cuda())
    pool = Fp32StatePool(plan, batch + 1, 64, get_format("fp32"))
    slots = torch.tensor([4, 0, 2, 1], device="cuda")
    state = torch.randn(batch, heads, keys, 64, device="cuda")
    pool.encode(state, slots)
    q = torch.randn(batch, heads, keys, device="cuda")
    k = torch.randn_like(q)
    v = torch.randn(batch, heads, 64, device="cuda")
    g = torch.randn(batch, heads, keys, device="cuda") if arch == "kda" else torch.randn(batch, heads, device="cuda")
    b = torch.randn(batch, heads, device="cuda")
    a_log = torch.rand(heads, device="cuda")
    dt = torch.zeros(heads * keys if arch == "kda" else heads, device="cuda")
    before = pool.decode(slots).cpu().numpy()
    out = pool.step(q, k, v, g, b, slots, normalize=True, scale=keys ** -0.5, a_log=a_log, dt_bias=dt)
    o_out, o_upd = O.delta_step(before, *O.prepare_inputs(q.cpu().numpy(), k.cpu().numpy(), g.cpu().numpy(),
                                                          b.cpu().numpy(), heads, kda=arch == "kda", normalize=True,
                                                          scale=keys ** -0.5, a_log=a_log.cpu().numpy(),
                                                          dt_bias=dt.cpu().numpy())[:2],
                                v.cpu().numpy(), *O.prepare_inputs(q.cpu().numpy(), k.cpu().numpy(), g.cpu().numpy(),
                                                                   b.cpu().numpy(), heads, kda=arch == "kda",
                                                                   normalize=True, scale=keys ** -0.5,
                                                                   a_log=a_log.cpu().numpy(),
                                                                   dt_bias=dt.cpu().numpy())[2:])
    active = slots.cpu().numpy() > 0
    torch.testing.assert_close(out.cpu()[active], torch.from_numpy(o_out)[active], atol=5e-5, rtol=1e-4)
    torch.testing.assert_close(pool.decode(slots).cpu()[active], torch.from_numpy(o_upd)[active], atol=5e-5, rtol=1e-4)
    assert out[1].count_nonzero() == 0
