"""KDA prefill (csrc/sq_prefill_kda.cu) against the token-by-token recurrence.

The kernel keeps the state in fp32 and applies core.delta_step token by token
with a per-key-channel decay, as the oracle's ``prefill_sequential`` does
(fp32, products summed in float64): the two differ only in summation order.
Final states within ``TOL_STATE`` of their largest magnitude; bf16 outputs
within one bf16 rounding step of theirs (``TOL_OUT``).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu

TOL_STATE = 1e-4
TOL_OUT = 8e-3


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _inputs(tokens, heads, qk_heads, gen, decay_scale=1.0):
    """KDA-shaped inputs: g = -exp(A_log) * softplus(u) per token, value head
    and key channel (the Kimi gate), beta = sigmoid."""
    q = torch.randn(tokens, qk_heads, 128, generator=gen).bfloat16()
    k = torch.randn(tokens, qk_heads, 128, generator=gen).bfloat16()
    v = torch.randn(tokens, heads, 128, generator=gen).bfloat16()
    a_log = torch.rand(heads, 1, generator=gen) * np.log(16)
    g = -a_log.exp() * torch.nn.functional.softplus(torch.randn(tokens, heads, 128, generator=gen)) * decay_scale
    beta = torch.randn(tokens, heads, generator=gen).sigmoid()
    return q, k, v, g, beta


def _check(out, final, q, k, v, g, beta, cu, init=None):
    o_ref, f_ref = O.prefill_sequential(q.float().numpy(), k.float().numpy(), v.float().numpy(), g.numpy(),
                                        beta.numpy(), cu, None if init is None else init.numpy())
    torch.cuda.synchronize()
    assert _rel(final.cpu().numpy(), f_ref) < TOL_STATE
    assert _rel(out.float().cpu().numpy(), o_ref) < TOL_OUT


@pytest.mark.parametrize("case", ["c", "d"])
def test_kda_prefill_matches_reference_recurrent_kernel(case):
    """Golden vectors of the reference's adapters.RecurrentKernel("kda") (150
    tokens from an initial state, 64 from zero)."""
    from stepquant_b200.kernels.prefill import chunk_kda
    d = load_golden("prefill.npz")
    q, k, v, g, beta = (torch.from_numpy(d[f"{case}_{n}"]).cuda() for n in ("q", "k", "v", "g", "beta"))
    init = torch.from_numpy(d[f"{case}_initial"]).cuda() if f"{case}_initial" in d else None
    out, final = chunk_kda(q.bfloat16(), k.bfloat16(), v.bfloat16(), g, beta, initial_state=init,
                           use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert out.shape == v.shape and out.dtype == torch.bfloat16
    assert _rel(final.cpu().numpy(), d[f"{case}_final"]) < TOL_STATE
    assert _rel(out.float().cpu().numpy(), d[f"{case}_out"]) < TOL_OUT


@pytest.mark.parametrize("decay_scale", [1.0, 0.01])
def test_kda_prefill_ragged_gqa_against_oracle(decay_scale):
    """Ragged sequences (an empty one, partial and exact 16-token blocks), GQA
    4 / 2, initial states; the empty sequence keeps its state exactly."""
    from stepquant_b200.kernels.prefill import chunk_kda
    gen = torch.Generator().manual_seed(31)
    heads, qk = 4, 2
    cu = [0, 70, 70, 198, 201, 265]
    q, k, v, g, beta = _inputs(cu[-1], heads, qk, gen, decay_scale)
    init = torch.randn(len(cu) - 1, heads, 128, 128, generator=gen) * 0.2
    out, final = chunk_kda(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), initial_state=init.cuda(),
                           cu_seqlens=torch.tensor(cu, dtype=torch.int32).cuda())
    assert out.shape == v.shape and out.dtype == torch.bfloat16
    _check(out, final, q, k, v, g, beta, cu, init)
    assert torch.equal(final[1].cpu(), init[1])


def test_kda_prefill_2048_token_prompts():
    """Config 3's prompt length with a slow decay (long memory): two prompts
    of 2,048 tokens from zero states, batched [1, T, H, K] inputs."""
    from stepquant_b200.kernels.prefill import chunk_kda
    gen = torch.Generator().manual_seed(32)
    heads, qk = 2, 1
    cu = [0, 2048, 4096]
    q, k, v, g, beta = _inputs(cu[-1], heads, qk, gen, 0.01)
    out, final = chunk_kda(q[None].cuda(), k[None].cuda(), v[None].cuda(), g[None].cuda(), beta[None].cuda(),
                           cu_seqlens=torch.tensor(cu, dtype=torch.int32).cuda())
    assert out.shape == (1,) + tuple(v.shape)
    _check(out[0], final, q, k, v, g, beta, cu)


def test_kda_prefill_unnormalised_and_scale():
    """use_qk_l2norm_in_kernel=False with an explicit scale against the oracle."""
    from stepquant_b200.kernels.prefill import chunk_kda
    gen = torch.Generator().manual_seed(33)
    heads, qk = 2, 2
    cu = [0, 37, 90]
    q, k, v, g, beta = _inputs(cu[-1], heads, qk, gen)
    q, k = (q.float() * 0.1).bfloat16(), (k.float() * 0.1).bfloat16()
    out, final = chunk_kda(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), scale=0.25,
                           use_qk_l2norm_in_kernel=False, cu_seqlens=torch.tensor(cu, dtype=torch.int32).cuda())
    o_ref, f_ref = O.prefill_sequential(q.float().numpy(), k.float().numpy(), v.float().numpy(), g.numpy(),
                                        beta.numpy(), cu, scale=0.25, normalize=False)
    torch.cuda.synchronize()
    assert _rel(final.cpu().numpy(), f_ref) < TOL_STATE
    assert _rel(out.float().cpu().numpy(), o_ref) < TOL_OUT


def test_kda_pool_extend_and_continuation():
    """PackedStatePool.extend on a KDA plan == decode -> chunk_kda -> encode,
    byte for byte; a prompt split in two passes equals one pass."""
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.prefill import chunk_kda
    gen = torch.Generator().manual_seed(34)
    heads, qk, tokens, split = 4, 4, 150, 61
    q, k, v, g, beta = (t.cuda() for t in _inputs(tokens, heads, qk, gen))
    _, whole = chunk_kda(q, k, v, g, beta)
    _, first = chunk_kda(q[:split], k[:split], v[:split], g[:split], beta[:split])
    _, second = chunk_kda(q[split:], k[split:], v[split:], g[split:], beta[split:], initial_state=first)
    assert _rel(second.cpu().numpy(), whole.cpu().numpy()) < TOL_STATE
    bits = torch.tensor([2, 4, 6, 16])[torch.randint(0, 4, (heads, 128), generator=gen)]
    plan = QuantizationPlan("kda", bits.cuda(), (torch.rand(heads, 128, generator=gen) + 0.5).cuda())
    pool, ref = PackedStatePool(plan, 3, 128), PackedStatePool(plan, 3, 128)
    slots = torch.tensor([2], device="cuda")
    state = torch.randn(1, heads, 128, 128, device="cuda") * 0.1
    pool.encode(state, slots)
    ref.encode(state, slots)
    cu = torch.tensor([0, tokens], device="cuda", dtype=torch.int32)
    out = pool.extend(q, k, v, g, beta, slots, cu)
    o2, fin = chunk_kda(q, k, v, g, beta, initial_state=ref.decode(slots), cu_seqlens=cu)
    ref.encode(fin, slots)
    assert torch.equal(out, o2) and torch.equal(pool.data, ref.data)


def test_kda_prefill_argument_errors():
    from stepquant_b200.kernels.prefill import chunk_kda
    q = torch.randn(10, 2, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(10, 2, 128, device="cuda", dtype=torch.bfloat16)
    beta = torch.rand(10, 2, device="cuda")
    with pytest.raises(ValueError):
        chunk_kda(q, q, v, beta, beta)  # a per-head g where KDA wants one per key channel
    with pytest.raises(ValueError):
        chunk_kda(q, q, v[:, :1].expand(10, 3, 128), torch.zeros(10, 3, 128, device="cuda"), beta)
