"""The CPU oracle against vectors produced by the unmodified reference.

These pin the oracle before it is trusted as the checker for the CUDA path:
``fit_state`` codes and fp16 scales, ``StateCodec`` byte streams, ``pack``,
``packed_layout`` tables, ``delta_step`` and the config-0 plumbing case must
all agree (bytes exactly; the fp32 recurrent update within 1e-5).
"""
import numpy as np
import pytest

from conftest import golden_fit_cases, load_golden, load_layouts
from oracle import stepquant_oracle as O


def _plan(d):
    return O.Plan(str(d["architecture"]), d["bits"].astype(np.int64), d["impact"], int(d["group"]))


def _same_bits(a, b):
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype == b.dtype and bool((a.view(np.uint8) == b.view(np.uint8)).all())


@pytest.mark.parametrize("case", golden_fit_cases())
def test_fit_state_matches_reference_bit_for_bit(case):
    d = load_golden(f"fit_{case}.npz")
    plan = _plan(d)
    z, r, c, r2, recon = O.fit_state(d["x"], plan)
    assert (z == d["z"]).all()
    assert _same_bits(r, d["r"])
    assert _same_bits(c, d["c"])
    if "r2" in d:
        assert _same_bits(r2, d["r2"])
    else:
        assert r2 is None
    # Pivot rows are exact fp16 copies.
    pivots = plan.bits == 16
    assert (recon[:, pivots] == d["x"][:, pivots].astype(np.float16).astype(np.float32)).all()


@pytest.mark.parametrize("case", golden_fit_cases())
def test_codec_streams_match_reference(case):
    d = load_golden(f"fit_{case}.npz")
    plan = _plan(d)
    enc = O.codec_encode(d["x"], plan)
    for b in (2, 4, 6, 8):
        assert _same_bits(enc["codes"][b], d[f"codes{b}"]), b
    assert _same_bits(enc["rows"], d["rows"])
    assert _same_bits(enc["columns"], d["columns"])
    assert _same_bits(enc["pivots"], d["pivots"])
    if "two_bit_rows" in d:
        assert _same_bits(enc["two_bit_rows"], d["two_bit_rows"])
    # decode(encode(x)) is fit_state's reconstruction (test_core.py:47-64).
    recon = O.fit_state(d["x"], plan)[-1]
    assert (O.codec_decode(enc, plan) == recon).all()


@pytest.mark.parametrize("case", golden_fit_cases())
def test_page_image_round_trip(case):
    d = load_golden(f"fit_{case}.npz")
    plan = _plan(d)
    pages = O.page_encode(d["x"], plan)
    assert pages.shape[1] == O.packed_layout(plan, d["x"].shape[-1])[-1]
    recon = O.fit_state(d["x"], plan)[-1]
    assert (O.page_decode(pages, plan, d["x"].shape[-1]) == recon).all()


def test_packed_layout_tables_match_reference():
    for entry in load_layouts():
        bits = np.array(entry["bits"])
        plan = O.Plan(entry["architecture"], bits, np.ones(bits.shape, np.float32), entry["value_group_size"])
        got = O.packed_layout(plan, entry["values"], entry["storage"])
        assert list(got) == [entry["offsets"], entry["rows"], entry["columns"], entry["page_bytes"]]


def test_byte_layout_known_answer():
    # test_byte_layout.py:9-20 of the reference, as a known-answer vector.
    bits = np.array([[2, 4, 6, 16], [16, 16, 16, 16]])
    plan = O.Plan("kda", bits, np.ones(bits.shape, np.float32))
    offsets, rows, columns, total = O.packed_layout(plan, 32, "byte")
    payload = 4 * 32 + 5 * 32 * 2
    assert offsets[8:] == [0, 192] and offsets[3] == 128
    assert columns == [payload + 3 * 2, -1]
    assert rows == [payload, payload + 2, payload + 4, -1, -1, -1, -1, -1]
    assert total == (payload + 3 * 2 + 32 * 2 + 15) // 16 * 16
    assert total > O.packed_layout(plan, 32, "packed")[-1]


@pytest.mark.parametrize("arch", ["gdn", "kda"])
def test_six_bit_page_has_no_padding(arch):
    # test_stepquant6.py:42-53: exactly H*K*V*6/8 + 2H(K+V) bytes.
    heads, keys, values = 2, 128, 128
    plan = O.Plan(arch, np.full((heads, keys), 6), np.ones((heads, keys), np.float32))
    assert O.packed_layout(plan, values)[-1] - 2 * heads * (keys + values) == heads * keys * values * 6 // 8


def test_half_aligned_mixed_kda_page():
    # test_kernel_edges.py:12-34: mixed KDA pages may be only half-aligned.
    plan = O.Plan("kda", np.array([[2, 4, 8, 16]]), np.ones((1, 4), np.float32))
    for values in (4, 32):
        assert O.packed_layout(plan, values)[-1] % 4 == 2


def test_pack_matches_reference():
    d = load_golden("pack.npz")
    for bits in (2, 4, 6, 8):
        for n in (0, 1, 7, 128, 513):
            codes = d[f"codes_{bits}_{n}"]
            packed = O.pack(codes, bits)
            assert _same_bits(packed, d[f"packed_{bits}_{n}"])
            assert (O.unpack(packed, bits, n) == codes).all()
            assert packed.size <= (n * bits + 7) // 8 + 2


def test_delta_step_matches_reference():
    d = load_golden("delta.npz")
    for arch in ("gdn", "kda"):
        g = {k: d[f"{arch}_{k}"] for k in ("state", "q", "k", "v", "g", "beta", "out", "updated")}
        out, updated = O.delta_step(g["state"], g["q"], g["k"], g["v"], g["g"], g["beta"])
        np.testing.assert_allclose(out, g["out"], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(updated, g["updated"], atol=1e-5, rtol=1e-5)


def test_config0_plumbing_case():
    """warm state, calibrated plan, one decode step, re-fit."""
    d = load_golden("config0.npz")
    plan = O.Plan("gdn", d["bits"].astype(np.int64), d["impact"], 32)
    z0, r0, c0, _, recon0 = O.fit_state(d["warm_state"], plan)
    assert (z0 == d["z0"]).all() and _same_bits(r0, d["r0"]) and _same_bits(c0, d["c0"])
    # The pool path: page image of the warm state, then one decode step.
    pages = O.page_encode(d["warm_state"], plan)
    slots = np.arange(1, 5)
    pool = np.zeros((5, pages.shape[1]), np.uint8)
    pool[1:] = pages
    out, new_pool, updated = O.decode_step(
        pool, slots, plan, 128, d["q"], d["k"], d["v"], d["a"], d["b"],
        normalize=True, scale=128 ** -0.5, a_log=d["a_log"], dt_bias=d["dt_bias"])
    np.testing.assert_allclose(out, d["out"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(updated, d["updated"], atol=2e-5, rtol=1e-4)
    # Codes are bit-exact given the same fp32 pre-quantization state.
    z, r, c, _, _ = O.fit_state(d["updated"], plan)
    assert (z == d["z"]).all() and _same_bits(r, d["r"]) and _same_bits(c, d["c"])
    assert (new_pool[0] == 0).all()


def test_zero_state_encodes_finite():
    bits = np.array([[2] * 8, [4] * 8, [6] * 8, [8] * 8, [16] * 8])
    for arch in ("gdn", "kda"):
        b = bits if arch == "gdn" else bits.T.copy()
        plan = O.Plan(arch, b, np.full(b.shape, 0.7, np.float32), 4)
        x = np.zeros((2,) + b.shape + (16,), np.float32)
        dec = O.codec_decode(O.codec_encode(x, plan), plan)
        assert np.isfinite(dec).all() and np.abs(dec).max() < 1e-10


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_prefill_oracle_matches_reference_recurrent_kernel(case):
    """oracle.prefill_sequential vs stepquant.adapters.RecurrentKernel (150 / 64
    tokens; a, b GDN with a decay per head, c, d KDA with one per key channel)."""
    d = load_golden("prefill.npz")
    q, k, v, g, beta = (d[f"{case}_{n}"][0] for n in ("q", "k", "v", "g", "beta"))
    init = d[f"{case}_initial"] if f"{case}_initial" in d else None
    out, final = O.prefill_sequential(q, k, v, g, beta, [0, q.shape[0]], init)
    np.testing.assert_allclose(final, d[f"{case}_final"], rtol=0, atol=1e-5 * np.abs(d[f"{case}_final"]).max())
    np.testing.assert_allclose(out, d[f"{case}_out"][0], rtol=0, atol=1e-5 * np.abs(d[f"{case}_out"]).max())


def test_byte_carrier_pages_hold_the_packed_levels():
    """storage='byte' pages (fit.py:111-115, byte_codec.py:6-27): the same
    fitted levels as packed pages, one int8 per value (KDA: times 2^(8-b)),
    contiguous fp16 pivot rows; both images decode to the same state."""
    rng = np.random.default_rng(5)
    for arch, bits in (("kda", np.array([[2, 4, 6, 16] * 8, [16] * 32])),
                       ("gdn", np.array([[4] * 32, [2] * 32, [16] * 32, [8] * 32]))):
        plan = O.Plan(arch, bits, (rng.random(bits.shape) + 0.5).astype(np.float32), 8)
        state = (rng.standard_normal((2, bits.shape[0], 32, 32)) * 0.1).astype(np.float32)
        byte_pages = O.page_encode(state, plan, storage="byte")
        packed_pages = O.page_encode(state, plan)
        assert byte_pages.shape[1] == O.packed_layout(plan, 32, "byte")[-1]
        np.testing.assert_array_equal(O.page_decode(byte_pages, plan, 32, "byte"), O.page_decode(packed_pages, plan, 32))
        z = O.fit_state(state, plan)[0]
        offsets = O.packed_layout(plan, 32, "byte")[0]
        code_base = offsets[bits.shape[0] * 32]
        k = 1 if arch == "kda" else 0  # a 4-bit row of head 0
        levels = byte_pages[0, code_base + k + np.arange(32) * 32].view(np.int8)
        expect = z[0, 0, k].astype(np.int64) * (16 if arch == "kda" else 1)
        np.testing.assert_array_equal(levels, expect)


@pytest.mark.parametrize("name", ["sym_int4_g128", "sym_int6_g128", "sym_int8_g128", "dsq_int4", "dsq_int6"])
def test_baseline_formats_match_reference(name):
    """formats.py group_fit / dual_fit and format_pool.format_layout of the
    reference (tests/golden/formats.npz) against the oracle's restatement;
    the oracle's page image decodes back to the reference reconstruction."""
    d = load_golden("formats.npz")
    x = d["x"]
    kind, bits, group = O.format_spec(name)
    if kind == "symmetric":
        codes, s, z, recon = O.group_fit(x, bits, group)
        np.testing.assert_array_equal(s, d[f"{name}_s"])
        np.testing.assert_array_equal(z, d[f"{name}_z"])
    else:
        codes, r, c, _, recon = O.dual_fit(x, bits)
        np.testing.assert_array_equal(r, d[f"{name}_r"])
        np.testing.assert_array_equal(c, d[f"{name}_c"])
    np.testing.assert_array_equal(codes, d[f"{name}_q"].astype(np.float32))
    np.testing.assert_array_equal(recon, d[f"{name}_recon"])
    heads, keys, values = x.shape[1:]
    offsets, rows, columns, total = O.format_layout(heads, keys, values, kind, bits, group)
    np.testing.assert_array_equal(np.array(offsets + rows + columns + [total]), d[f"{name}_layout"])
    pages = O.format_page_encode(x, name)
    assert pages.shape == (x.shape[0], total)
    np.testing.assert_array_equal(O.format_page_decode(pages, name, heads, keys, values), d[f"{name}_recon"])


def _extension_cases():
    d = load_golden("widths_ext.npz")
    return sorted({k.rsplit("_", 1)[0] for k in d.files if k.endswith("_arch")})


@pytest.mark.parametrize("case", _extension_cases())
def test_extended_widths_fit_state_matches_reference_formula(case):
    """3- and 5-bit rows (this build's extension): the oracle's fit_state equals
    the reference's own fit_state run on a plan built without its width
    validation (tests/golden/make_golden.py --extension-only)."""
    d = load_golden("widths_ext.npz")
    plan = O.Plan(str(d[f"{case}_arch"]), d[f"{case}_bits"].astype(np.int64), d[f"{case}_impact"],
                  int(d[f"{case}_group"]), extended_widths=True)
    z, r, c, r2, recon = O.fit_state(d[f"{case}_x"], plan)
    assert (z == d[f"{case}_z"]).all()
    assert _same_bits(r, d[f"{case}_r"]) and _same_bits(c, d[f"{case}_c"])
    # decode(encode(x)) through the extended codec and page image is the reconstruction.
    enc = O.codec_encode(d[f"{case}_x"], plan)
    assert (O.codec_decode(enc, plan) == recon).all()
    pages = O.page_encode(d[f"{case}_x"], plan)
    assert (O.page_decode(pages, plan, d[f"{case}_x"].shape[-1]) == recon).all()


def test_extended_widths_are_opt_in():
    bits = np.full((2, 8), 3)
    with pytest.raises(ValueError):
        O.Plan("kda", bits, np.ones((2, 8), np.float32))
    with pytest.raises(ValueError):
        O.pack(np.zeros(8, np.int64), 3)
    for b in (3, 5):
        codes = np.random.default_rng(b).integers(0, 2 ** b, 37)
        data = O.pack(codes, b, extended=True)
        assert data.size == (37 + 7) // 8 * b
        assert (O.unpack(data, b, 37) == codes).all()
    # KDA value tiles of 4: a 3-bit row takes 2 bytes per tile, a 5-bit row 3.
    plan = O.Plan("kda", np.array([[3, 5, 16, 4]]), np.ones((1, 4), np.float32), extended_widths=True)
    offsets, rows, columns, total = O.packed_layout(plan, 8)
    assert offsets[:4] == [0, 2, 6, 14] and offsets[4] == 16  # the pivot row: 4 fp16 values per tile
