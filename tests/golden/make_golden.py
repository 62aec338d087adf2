"""Generate golden vectors from the unmodified reference STEPQuant (torch CPU path).

Run from the repository root in a container where the reference checkout is
available (its path is given by ``--reference``):

    python tests/golden/make_golden.py --reference <path to the STEPQuant checkout>

The GPU box never runs this script; tests read the committed ``*.npz`` /
``layouts.json`` files only.  Everything is seeded.  torch runs with one
thread, although the reference's sums give identical bits with eight.

Files written next to this script:
* ``layouts.json``   -- ``stepquant.kernels.pool.packed_layout`` tables.
* ``fit_<case>.npz`` -- ``stepquant.quantization.fit_state`` outputs and the
                        ``StateCodec.encode`` byte streams for a seeded state.
* ``pack.npz``       -- ``stepquant.packing.pack`` outputs.
* ``delta.npz``      -- ``stepquant.core.delta_step`` outputs.
* ``config0.npz``    -- the CPU reference plumbing case (GDN, B=4, H=HK=4,
                        K=V=128, seed 0): warm-up state, calibrated plan,
                        decode inputs, the updated state and its fitted codes.
* ``prefill.npz``    -- ``stepquant.adapters.RecurrentKernel`` (the token-by-
                        token prefill recurrence) on bf16-valued q/k/v with
                        in-kernel L2 normalisation: outputs and final states;
                        cases a, b GDN (decay per head), c, d KDA (decay per
                        key channel).

* ``calibration.npz`` -- ``stepquant.calibration``: the statistics a seeded
                        run of ``LayerStatistics.observe`` exports (two GDN
                        and two KDA layers), the plans ``calibrate`` makes from
                        them, and ``stepquant.allocation`` on seeded cost
                        tables.

* ``formats.npz``  -- ``stepquant.formats`` baseline formats (sym_int*_g128
                        ``group_fit``, dsq_int* ``dual_fit``) on seeded states,
                        and ``kernels.format_pool.format_layout`` tables.

* ``widths_ext.npz`` -- ``stepquant.quantization.fit_state`` at 3- and 5-bit
                        rows (this build's width extension; the reference's
                        QuantizationPlan rejects those widths, so the plan
                        object is built without its validation and fit_state,
                        whose formula is width-generic, runs unchanged).

``--extension-only`` rewrites ``widths_ext.npz`` alone;
``--prefill-only`` rewrites ``prefill.npz`` alone; ``--calibration-only``
rewrites ``calibration.npz`` alone; ``--formats-only`` rewrites
``formats.npz`` alone.
"""
import argparse
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits_mixed(arch, heads_bits, keys):
    bits = torch.tensor(heads_bits)[:, None].expand(len(heads_bits), keys).clone()
    return bits


def fit_cases():
    """(name, arch, bits[H,K], group, batch, values, scale, seed)."""
    cases = []
    g5 = [2, 4, 6, 8, 16]
    cases.append(("gdn_mixed_k32", "gdn", _bits_mixed("gdn", g5, 32), 32, 2, 32, 1.0, 31))
    cases.append(("gdn_mixed_k32_g8", "gdn", _bits_mixed("gdn", g5, 32), 8, 2, 32, 1.0, 32))
    kb = _bits_mixed("kda", g5, 32).roll(1, 0)
    kb[:, ::3] = 16
    kb[:, 1::4] = 2
    cases.append(("kda_mixed_k32", "kda", kb, 32, 2, 32, 1.0, 33))
    cases.append(("gdn_k128", "gdn", _bits_mixed("gdn", [4, 6, 8, 16, 2], 128), 32, 2, 128, 0.1, 34))
    gen = torch.Generator().manual_seed(35)
    kb = torch.tensor([2, 4, 6, 8])[torch.randint(0, 4, (3, 128), generator=gen)]
    kb[torch.rand(3, 128, generator=gen) < 0.05] = 16
    cases.append(("kda_k128", "kda", kb, 32, 2, 128, 0.1, 36))
    cases.append(("gdn_k128_v64", "gdn", _bits_mixed("gdn", [4, 6, 8, 2], 128), 32, 2, 64, 0.1, 37))
    cases.append(("gdn_k128_v16", "gdn", _bits_mixed("gdn", [4, 6, 8, 2], 128), 16, 2, 16, 0.1, 38))
    cases.append(("kda_k64_v8", "kda", torch.tensor([4, 6, 8, 16, 2])[torch.randint(0, 5, (2, 64), generator=gen)], 32, 3, 8, 1.0, 39))
    cases.append(("gdn_k4_v8", "gdn", _bits_mixed("gdn", g5, 4), 8, 2, 8, 1.0, 40))
    cases.append(("kda_k4_v4_half", "kda", torch.tensor([[2, 4, 8, 16]]), 32, 3, 4, 1.0, 41))
    cases.append(("kda_k16_v32", "kda", torch.tensor([[4, 6, 8] * 5 + [16]] * 2), 32, 2, 32, 1.0, 42))
    return cases


def layout_cases():
    cases = []
    cases.append(("kda", [[2, 4, 6, 16], [16, 16, 16, 16]], 32, 32))
    cases.append(("kda", [[2, 4, 8, 16]], 4, 32))
    cases.append(("kda", [[2, 4, 8, 16]], 32, 32))
    cases.append(("gdn", [[b] * 4 for b in (2, 4, 6, 8, 16)], 8, 8))
    cases.append(("gdn", [[6] * 128] * 2, 128, 32))
    cases.append(("kda", [[6] * 128] * 2, 128, 32))
    gen = torch.Generator().manual_seed(11)
    widths = [4] * 8 + [6] * 16 + [8] * 8
    perm = torch.randperm(32, generator=gen).tolist()
    cases.append(("gdn", [[widths[i]] * 128 for i in perm], 128, 32))
    cases.append(("gdn", [[widths[i] if n else 16] * 128 for n, i in enumerate(perm)], 128, 32))
    kb = torch.tensor([2, 4, 6])[torch.multinomial(torch.tensor([.3, .5, .2]), 32 * 128, True, generator=gen)].reshape(32, 128)
    kb[torch.rand(32, 128, generator=gen) < 0.02] = 16
    cases.append(("kda", kb.tolist(), 128, 32))
    return cases


def prefill_cases(RecurrentKernel):
    """Two sequences' worth of seeded prompts through the reference recurrence."""
    out = {}
    gen = torch.Generator().manual_seed(3)
    for name, tokens, initial in (("a", 150, True), ("b", 64, False)):
        heads, keys, values = 2, 128, 128
        q = torch.randn(1, tokens, heads, keys, generator=gen).bfloat16().float()
        k = torch.randn(1, tokens, heads, keys, generator=gen).bfloat16().float()
        v = torch.randn(1, tokens, heads, values, generator=gen).bfloat16().float()
        a_log = torch.rand(heads, generator=gen) * math.log(16)
        g = -a_log.exp() * torch.nn.functional.softplus(torch.randn(1, tokens, heads, generator=gen))
        beta = torch.randn(1, tokens, heads, generator=gen).sigmoid()
        state = torch.randn(1, heads, keys, values, generator=gen) * 0.1 if initial else None
        o, final = RecurrentKernel("gdn")(q, k, v, g, beta, initial_state=state, output_final_state=True,
                                          use_qk_l2norm_in_kernel=True)
        out.update({f"{name}_{n}": t.numpy() for n, t in dict(q=q, k=k, v=v, g=g, beta=beta, out=o, final=final).items()})
        if initial:
            out[f"{name}_initial"] = state.numpy()
    # KDA (per-key-channel decay, the Kimi gate -exp(A_log) softplus(.) per
    # channel): the same recurrence with g [1, T, H, K]; GQA-free, 2 heads.
    gen = torch.Generator().manual_seed(4)
    for name, tokens, initial in (("c", 150, True), ("d", 64, False)):
        heads, keys, values = 2, 128, 128
        q = torch.randn(1, tokens, heads, keys, generator=gen).bfloat16().float()
        k = torch.randn(1, tokens, heads, keys, generator=gen).bfloat16().float()
        v = torch.randn(1, tokens, heads, values, generator=gen).bfloat16().float()
        a_log = torch.rand(heads, 1, generator=gen) * math.log(16)
        g = -a_log.exp() * torch.nn.functional.softplus(torch.randn(1, tokens, heads, keys, generator=gen))
        beta = torch.randn(1, tokens, heads, generator=gen).sigmoid()
        state = torch.randn(1, heads, keys, values, generator=gen) * 0.1 if initial else None
        o, final = RecurrentKernel("kda")(q, k, v, g, beta, initial_state=state, output_final_state=True,
                                          use_qk_l2norm_in_kernel=True)
        out.update({f"{name}_{n}": t.numpy() for n, t in dict(q=q, k=k, v=v, g=g, beta=beta, out=o, final=final).items()})
        if initial:
            out[f"{name}_initial"] = state.numpy()
    return out


CALIBRATION_CASES = (  # (arch, layers, heads, keys, values, nominal bits, pivots, seed)
    ("gdn", 2, 6, 32, 32, 6, 2, 41),
    ("kda", 2, 2, 32, 32, 4, 8, 42),
)


def observe_run(LayerStatistics, arch, heads, keys, values, seed, updates=32, batch=4):
    """A seeded stream of observe() calls (tests/test_calibration.py replays
    it); returns the exported statistics."""
    gen = torch.Generator().manual_seed(seed)
    stat = LayerStatistics(arch, sample_every=8, max_snapshots=6)
    for _ in range(updates):
        q = torch.randn(batch, heads, keys, generator=gen)
        k = torch.nn.functional.normalize(torch.randn(batch, heads, keys, generator=gen), dim=-1)
        v = torch.randn(batch, heads, values, generator=gen)
        shape = (batch, heads) if arch == "gdn" else (batch, heads, keys)
        log_decay = -torch.rand(shape, generator=gen) * 0.2
        beta = torch.rand(batch, heads, generator=gen)
        state = torch.randn(batch, heads, keys, values, generator=gen) * 0.1
        stat.observe(q, k, v, log_decay, beta, state)
    return stat.export()


def calibration_vectors(reference_modules):
    LayerStatistics, calibrate, allocate_dp, allocate_lagrangian = reference_modules
    out = {}
    for arch, layers, heads, keys, values, nominal, pivots, seed in CALIBRATION_CASES:
        stats = {}
        for layer in range(layers):
            name = f"model.layers.{3 * layer}.mixer"
            stats[name] = observe_run(LayerStatistics, arch, heads, keys, values, seed + 100 * layer)
            e = stats[name]
            for key in ("omega", "log_decay", "snapshots"):
                out[f"{arch}_{layer}_{key}"] = e[key].numpy()
            out[f"{arch}_{layer}_counts"] = np.array([e["tokens"], e["sampled_states"]])
        result = calibrate(stats, nominal_bits=nominal, pivots=pivots, horizon=256, value_group_size=8)
        for layer, name in enumerate(sorted(stats)):
            out[f"{arch}_{layer}_bits"] = result["plans"][name]["bits"].numpy().astype(np.int8)
            out[f"{arch}_{layer}_impact"] = result["plans"][name]["impact"].numpy()
        st = result["settings"]
        out[f"{arch}_budget"] = np.array([st["integer_budget"], st["integer_bits_used"]])
    gen = torch.Generator().manual_seed(43)
    for name, fn, units in (("dp", allocate_dp, 24), ("lagrangian", allocate_lagrangian, 200)):
        candidates = [4, 6, 8] if name == "dp" else [2, 4, 6, 8]
        cost = torch.rand(units, len(candidates), generator=gen).double()
        cost = torch.sort(cost, dim=1, descending=True).values  # wider is better, mostly
        cost[::7] = torch.rand(len(cost[::7]), len(candidates), generator=gen).double()  # some non-monotone rows
        budget = int(units * (5 if name == "dp" else 4))
        out[f"alloc_{name}_cost"] = cost.numpy()
        out[f"alloc_{name}_budget"] = np.array(budget)
        out[f"alloc_{name}_result"] = fn(cost, candidates, budget).numpy()
    return out


FORMAT_CASES = ("sym_int4_g128", "sym_int6_g128", "sym_int8_g128", "dsq_int4", "dsq_int6")


def format_vectors(get_format, group_fit, dual_fit, format_layout):
    """Baseline-format fits of one seeded state [2, 2, 16, 128] and their page layouts."""
    gen = torch.Generator().manual_seed(44)
    heads, keys, values = 2, 16, 128
    x = torch.randn(2, heads, keys, values, generator=gen) * 0.1
    x[1, 0, 3] = 0  # an all-zero row
    x[1, 1, :, 7] *= 40  # a large column
    out = {"x": x.numpy()}
    for name in FORMAT_CASES:
        spec = get_format(name)
        bits = torch.full((heads, keys), spec.bits, dtype=torch.long)
        impact = torch.rand(heads, keys, generator=gen) + 0.5
        if spec.kind == "symmetric":
            q, scale, zero, recon = group_fit(x, spec)
            out[f"{name}_q"] = q.numpy().astype(np.uint8)
            out[f"{name}_s"] = scale.numpy()
            out[f"{name}_z"] = zero.numpy()
        else:
            q, r, c, zero, recon = dual_fit(x, bits, impact)
            out[f"{name}_q"] = q.numpy().astype(np.uint8)
            out[f"{name}_r"] = r.numpy()
            out[f"{name}_c"] = c.numpy()
        out[f"{name}_recon"] = recon.numpy()

        class _Plan:  # format_layout reads plan.bits only
            pass
        plan = _Plan()
        plan.bits = bits
        offsets, rows, columns, total = format_layout(plan, values, spec)
        out[f"{name}_layout"] = np.array(offsets + rows + columns + [total], dtype=np.int64)
    return out


def extension_cases():
    """(name, arch, bits[H,K], group, batch, values, scale, seed) with 3/5-bit rows."""
    gen = torch.Generator().manual_seed(50)
    kda = torch.tensor([3, 4, 6])[torch.multinomial(torch.tensor([0.3, 0.5, 0.2]), 2 * 128, True, generator=gen)]
    kda = kda.reshape(2, 128)
    kda[torch.rand(2, 128, generator=gen) < 0.02] = 16
    return [
        ("gdn_w35_k32", "gdn", _bits_mixed("gdn", [3, 5, 4, 6, 8, 16], 32), 32, 2, 32, 1.0, 51),
        ("gdn_w35_k128", "gdn", _bits_mixed("gdn", [3, 5, 6], 128), 32, 1, 128, 0.1, 52),
        ("kda_w346_k128", "kda", kda, 32, 1, 128, 0.1, 53),
        ("kda_w35_k16", "kda", torch.tensor([[3, 5, 16, 4] * 4, [5, 3, 8, 2] * 4]), 32, 3, 8, 1.0, 54),
    ]


def extension_vectors(QuantizationPlan, fit_state):
    out = {}
    for name, arch, bits, group, batch, values, scale, seed in extension_cases():
        torch.manual_seed(seed)
        heads, keys = bits.shape
        impact = torch.rand(heads, keys) + 0.25
        plan = object.__new__(QuantizationPlan)  # no width validation: 3/5 bits are this build's extension
        plan.architecture, plan.bits, plan.impact, plan.value_group_size = arch, bits, impact, group
        x = torch.randn(batch, heads, keys, values) * scale
        z, r, c, r2, recon = fit_state(x, plan)
        out.update({f"{name}_arch": np.array(arch), f"{name}_bits": bits.numpy().astype(np.int8),
                    f"{name}_impact": impact.numpy(), f"{name}_group": np.array(group), f"{name}_x": x.numpy(),
                    f"{name}_z": z.numpy().astype(np.int8), f"{name}_r": r.numpy(), f"{name}_c": c.numpy()})
    return out


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the STEPQuant checkout")
    parser.add_argument("--prefill-only", action="store_true")
    parser.add_argument("--calibration-only", action="store_true")
    parser.add_argument("--formats-only", action="store_true")
    parser.add_argument("--extension-only", action="store_true")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    if args.extension_only:
        from stepquant.quantization import QuantizationPlan, fit_state
        torch.set_num_threads(1)
        np.savez_compressed(os.path.join(HERE, "widths_ext.npz"), **extension_vectors(QuantizationPlan, fit_state))
        print("extension vectors written to", HERE)
        return
    if args.formats_only:
        from stepquant.formats import get_format, group_fit, dual_fit
        from stepquant.kernels.format_pool import format_layout
        torch.set_num_threads(1)
        np.savez_compressed(os.path.join(HERE, "formats.npz"),
                            **format_vectors(get_format, group_fit, dual_fit, format_layout))
        print("format vectors written to", HERE)
        return
    if args.calibration_only:
        from stepquant.calibration import LayerStatistics, calibrate
        from stepquant.allocation import allocate_dp, allocate_lagrangian
        torch.set_num_threads(1)
        np.savez_compressed(os.path.join(HERE, "calibration.npz"),
                            **calibration_vectors((LayerStatistics, calibrate, allocate_dp, allocate_lagrangian)))
        print("calibration vectors written to", HERE)
        return
    if args.prefill_only:
        from stepquant.adapters import RecurrentKernel
        torch.set_num_threads(1)
        np.savez_compressed(os.path.join(HERE, "prefill.npz"), **prefill_cases(RecurrentKernel))
        print("prefill vectors written to", HERE)
        return
    torch.set_num_threads(1)
    from stepquant.quantization import QuantizationPlan, StateCodec, fit_state
    from stepquant.packing import pack
    from stepquant.core import delta_step, impact_factors
    from stepquant.calibration import LayerStatistics
    from stepquant.kernels.pool import packed_layout

    layouts = []
    for arch, bits, values, group in layout_cases():
        b = torch.tensor(bits)
        plan = QuantizationPlan(arch, b, torch.ones_like(b).float(), group)
        for storage in ("packed", "byte"):
            offsets, rows, columns, total = packed_layout(plan, values, storage)
            layouts.append(dict(architecture=arch, bits=bits, values=values, value_group_size=group,
                                storage=storage, offsets=offsets, rows=rows, columns=columns,
                                page_bytes=total))
    with open(os.path.join(HERE, "layouts.json"), "w") as fh:
        json.dump(layouts, fh, separators=(",", ":"))

    for name, arch, bits, group, batch, values, scale, seed in fit_cases():
        torch.manual_seed(seed)
        heads, keys = bits.shape
        impact = torch.rand(heads, keys) + 0.25
        plan = QuantizationPlan(arch, bits, impact, group)
        x = torch.randn(batch, heads, keys, values) * scale
        if name == "gdn_k4_v8":
            x[1] = 0  # an all-zero request
        z, r, c, r2, recon = fit_state(x, plan)
        packed = StateCodec(plan).encode(x)
        out = dict(architecture=np.array(arch), bits=bits.numpy().astype(np.int8), impact=impact.numpy(),
                   group=np.array(group), x=x.numpy(), z=z.numpy().astype(np.int8), r=r.numpy(), c=c.numpy(),
                   rows=packed.rows.numpy(), columns=packed.columns.numpy(),
                   pivots=packed.pivots.numpy())
        if r2 is not None:
            out["r2"] = r2.numpy()
            out["two_bit_rows"] = packed.two_bit_rows.numpy()
        for b, stream in packed.codes.items():
            out[f"codes{b}"] = stream.numpy()
        np.savez_compressed(os.path.join(HERE, f"fit_{name}.npz"), **out)

    torch.manual_seed(5)
    packs = {}
    for bits in (2, 4, 6, 8):
        for n in (0, 1, 7, 128, 513):
            codes = torch.randint(2 ** bits, (n,))
            packs[f"codes_{bits}_{n}"] = codes.numpy().astype(np.int16)
            packs[f"packed_{bits}_{n}"] = pack(codes, bits).numpy()
    np.savez_compressed(os.path.join(HERE, "pack.npz"), **packs)

    torch.manual_seed(2)
    deltas = {}
    for arch in ("gdn", "kda"):
        b, h, k, v = 3, 4, 16, 8
        state = torch.randn(b, h, k, v)
        q = torch.randn(b, h, k)
        key = torch.nn.functional.normalize(torch.randn(b, h, k), dim=-1)
        val, beta = torch.randn(b, h, v), torch.rand(b, h)
        g = -torch.rand(b, h) if arch == "gdn" else -torch.rand(b, h, k)
        y, s = delta_step(state, q, key, val, g, beta)
        deltas.update({f"{arch}_{n}": t.numpy() for n, t in
                       dict(state=state, q=q, k=key, v=val, g=g, beta=beta, out=y, updated=s).items()})
    np.savez_compressed(os.path.join(HERE, "delta.npz"), **deltas)

    # Config 0: CPU reference plumbing.
    gen = torch.Generator().manual_seed(0)
    batch, heads, qk_heads, keys, values = 4, 4, 4, 128, 128

    def draw_inputs():
        q = torch.randn(batch, qk_heads, keys, generator=gen)
        k = torch.randn(batch, qk_heads, keys, generator=gen)
        v = torch.randn(batch, heads, values, generator=gen).bfloat16()
        a = torch.randn(batch, heads, generator=gen)
        b = torch.randn(batch, heads, generator=gen)
        return q, k, v, a, b

    a_log = torch.rand(heads, generator=gen) * math.log(16)
    dt_bias = torch.zeros(heads)

    def prepare(q, k, a, b):
        qn = q * torch.rsqrt(q.square().sum(-1, keepdim=True) + 1e-6) * keys ** -0.5
        kn = k * torch.rsqrt(k.square().sum(-1, keepdim=True) + 1e-6)
        g = -a_log.exp() * torch.nn.functional.softplus(a + dt_bias)
        return qn.repeat_interleave(heads // qk_heads, 1), kn.repeat_interleave(heads // qk_heads, 1), g, b.sigmoid()

    stats = LayerStatistics("gdn", sample_every=64, max_snapshots=8)
    state = torch.zeros(batch, heads, keys, values)
    for _ in range(256):
        q, k, v, a, b = draw_inputs()
        qn, kn, g, beta = prepare(q, k, a, b)
        _, state = delta_step(state, qn, kn, v.float(), g, beta)
        stats.observe(qn, kn, v.float(), g, beta, state)
    impact = impact_factors(stats.export()["omega"])
    widths = torch.tensor([4, 6, 6, 8])[torch.randperm(heads, generator=gen)]
    bits = widths[:, None].expand(heads, keys).clone()
    plan = QuantizationPlan("gdn", bits, impact, 32)
    codec = StateCodec(plan)
    packed = codec.encode(state)
    decoded = codec.decode(packed)
    q, k, v, a, b = draw_inputs()
    qn, kn, g, beta = prepare(q, k, a, b)
    out, updated = delta_step(decoded, qn, kn, v.float(), g, beta)
    z, r, c, _, recon = fit_state(updated, plan)
    z0, r0, c0, _, _ = fit_state(state, plan)
    np.savez_compressed(
        os.path.join(HERE, "config0.npz"), bits=bits.numpy().astype(np.int8), impact=impact.numpy(),
        warm_state=state.numpy(), z0=z0.numpy().astype(np.int8), r0=r0.numpy(), c0=c0.numpy(),
        q=q.numpy(), k=k.numpy(), v=v.float().numpy(), a=a.numpy(), b=b.numpy(),
        a_log=a_log.numpy(), dt_bias=dt_bias.numpy(), out=out.numpy(), updated=updated.numpy(),
        z=z.numpy().astype(np.int8), r=r.numpy(), c=c.numpy())
    from stepquant.adapters import RecurrentKernel
    np.savez_compressed(os.path.join(HERE, "prefill.npz"), **prefill_cases(RecurrentKernel))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
