"""GDN chunked prefill (csrc/sq_prefill.cu) against the token-by-token recurrence.

The chunk pass multiplies bf16 operands on tensor cores (fp32 accumulation,
fp32 state), the reference recurrence runs in fp32, so parity is a tolerance:
the final state and the outputs within 2e-2 of their largest magnitude
(``TOL``) -- the same order as the reference's own prefill check after
quantization (tests/test_sglang_cuda.py: atol 5e-3 / rtol 1.5e-2).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import stepquant_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("case", ["a", "b"])
def test_prefill_matches_reference_recurrent_kernel(case):
    """Golden vectors of the reference's adapters.RecurrentKernel (150 and 64 tokens)."""
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule
    d = load_golden("prefill.npz")
    q, k, v, g, beta = (torch.from_numpy(d[f"{case}_{n}"]).cuda() for n in ("q", "k", "v", "g", "beta"))
    init = torch.from_numpy(d[f"{case}_initial"]).cuda() if f"{case}_initial" in d else None
    out, final = chunk_gated_delta_rule(q.bfloat16(), k.bfloat16(), v.bfloat16(), g, beta, initial_state=init,
                                        use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert out.shape == v.shape and out.dtype == torch.bfloat16
    assert _rel(final.cpu().numpy(), d[f"{case}_final"]) < TOL
    assert _rel(out.float().cpu().numpy(), d[f"{case}_out"]) < TOL


def _inputs(tokens, heads, qk_heads, gen, decay_scale=1.0):
    q = torch.randn(tokens, qk_heads, 128, generator=gen).bfloat16()
    k = torch.randn(tokens, qk_heads, 128, generator=gen).bfloat16()
    v = torch.randn(tokens, heads, 128, generator=gen).bfloat16()
    a_log = torch.rand(heads, generator=gen) * np.log(16)
    g = -a_log.exp() * torch.nn.functional.softplus(torch.randn(tokens, heads, generator=gen)) * decay_scale
    beta = torch.randn(tokens, heads, generator=gen).sigmoid()
    return q, k, v, g, beta


@pytest.mark.parametrize("decay_scale", [1.0, 0.01])
def test_prefill_variable_lengths_gqa_against_oracle(decay_scale):
    """Ragged sequences (an empty one, a partial last chunk, exact chunks), GQA, initial states."""
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule
    gen = torch.Generator().manual_seed(7)
    heads, qk = 4, 2
    cu = [0, 70, 70, 198, 201, 265]
    q, k, v, g, beta = _inputs(cu[-1], heads, qk, gen, decay_scale)
    init = torch.randn(len(cu) - 1, heads, 128, 128, generator=gen) * 0.2
    out, final = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), initial_state=init.cuda(),
                                        cu_seqlens=torch.tensor(cu, dtype=torch.int32).cuda())
    o_ref, f_ref = O.prefill_sequential(q.float().numpy(), k.float().numpy(), v.float().numpy(), g.numpy(),
                                        beta.numpy(), cu, init.numpy())
    torch.cuda.synchronize()
    assert _rel(final.cpu().numpy(), f_ref) < TOL
    assert _rel(out.float().cpu().numpy(), o_ref) < TOL
    assert torch.equal(final[1].cpu(), init[1])  # the empty sequence keeps its state


@pytest.mark.parametrize("decay_scale", [1.0, 0.01])
def test_prefill_2048_token_prompts(decay_scale):
    """BASELINE config 3's prompt length: two prompts of 2,048 tokens (32
    chunks each, so the state pass runs its full chunk chain), GQA 4 / 2, from
    zero states.  Final state and outputs within ``TOL`` of their largest
    magnitude, and the bf16 outputs within 2e-2 absolute (the stated output
    tolerance)."""
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule
    gen = torch.Generator().manual_seed(13)
    heads, qk = 4, 2
    cu = [0, 2048, 4096]
    q, k, v, g, beta = _inputs(cu[-1], heads, qk, gen, decay_scale)
    out, final = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(),
                                        cu_seqlens=torch.tensor(cu, dtype=torch.int32).cuda())
    o_ref, f_ref = O.prefill_sequential(q.float().numpy(), k.float().numpy(), v.float().numpy(), g.numpy(),
                                        beta.numpy(), cu)
    torch.cuda.synchronize()
    o = out.float().cpu().numpy()
    assert _rel(final.cpu().numpy(), f_ref) < TOL
    assert _rel(o, o_ref) < TOL
    assert np.abs(o - o_ref).max() <= 2e-2


def test_prefill_many_short_sequences():
    """More sequences than the offsets kernel has threads (1,300 of 0-70 tokens,
    many empty): every chunk finds its sequence and first token in the
    per-chunk table, and empty sequences keep their initial state."""
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule
    gen = torch.Generator().manual_seed(11)
    heads, qk, seqs = 2, 1, 1300
    lengths = torch.randint(0, 4, (seqs,), generator=gen)
    lengths[::97] = 70  # a few sequences longer than one chunk
    cu = [0] + torch.cumsum(lengths, 0).tolist()
    q, k, v, g, beta = _inputs(cu[-1], heads, qk, gen, 1.0)
    init = torch.randn(seqs, heads, 128, 128, generator=gen) * 0.2
    out, final = chunk_gated_delta_rule(q.cuda(), k.cuda(), v.cuda(), g.cuda(), beta.cuda(), initial_state=init.cuda(),
                                        cu_seqlens=torch.tensor(cu, dtype=torch.int32).cuda())
    o_ref, f_ref = O.prefill_sequential(q.float().numpy(), k.float().numpy(), v.float().numpy(), g.numpy(),
                                        beta.numpy(), cu, init.numpy())
    torch.cuda.synchronize()
    assert _rel(final.cpu().numpy(), f_ref) < TOL
    assert _rel(out.float().cpu().numpy(), o_ref) < TOL
    empty = (lengths == 0).nonzero().flatten()
    assert len(empty) > 0 and torch.equal(final[empty].cpu(), init[empty])


def test_prefill_continuation_and_pool_extend():
    """A prompt split in two passes (state carried through the pool) equals one pass."""
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule
    gen = torch.Generator().manual_seed(11)
    heads, qk, tokens, split = 4, 4, 200, 77
    q, k, v, g, beta = (t.cuda() for t in _inputs(tokens, heads, qk, gen))
    _, whole = chunk_gated_delta_rule(q, k, v, g, beta)
    _, first = chunk_gated_delta_rule(q[:split], k[:split], v[:split], g[:split], beta[:split])
    _, second = chunk_gated_delta_rule(q[split:], k[split:], v[split:], g[split:], beta[split:], initial_state=first)
    assert _rel(second.cpu().numpy(), whole.cpu().numpy()) < TOL
    # PackedStatePool.extend == decode -> chunk pass -> encode, byte for byte.
    bits = torch.tensor([4, 6, 8, 6])[:, None].expand(heads, 128).clone()
    plan = QuantizationPlan("gdn", bits.cuda(), (torch.rand(heads, 128, generator=gen) + 0.5).cuda())
    pool, ref = PackedStatePool(plan, 3, 128), PackedStatePool(plan, 3, 128)
    slots = torch.tensor([2], device="cuda")
    cu = torch.tensor([0, tokens], device="cuda", dtype=torch.int32)
    out = pool.extend(q, k, v, g, beta, slots, cu)
    o2, fin = chunk_gated_delta_rule(q, k, v, g, beta, initial_state=ref.decode(slots), cu_seqlens=cu)
    ref.encode(fin, slots)
    assert torch.equal(out, o2) and torch.equal(pool.data, ref.data)


def test_prefill_argument_errors():
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule
    q = torch.randn(10, 2, 128, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(10, 3, 128, device="cuda", dtype=torch.bfloat16)
    g = torch.zeros(10, 3, device="cuda")
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(q, q, v, g, g)  # 3 value heads over 2 qk heads
    with pytest.raises(NotImplementedError):
        x = torch.randn(10, 2, 64, device="cuda", dtype=torch.bfloat16)
        chunk_gated_delta_rule(x, x, x, g[:, :2], g[:, :2])
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(q.cpu(), q.cpu(), v[:, :2].cpu(), g[:, :2].cpu(), g[:, :2].cpu())
