"""Host-side logic that needs no GPU: the C ABI library, page layout, plan
validation, format registry, writeback profiles and the release schedule."""
import ctypes
import os
import re
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import ROOT, load_layouts


def _header_symbols():
    text = open(os.path.join(ROOT, "include", "stepquant_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(sq_\w+)\s*\(", text, re.M)))


def test_library_loads_and_exports_every_declared_symbol():
    from stepquant_b200 import _native as N
    lib = N.lib()
    declared = _header_symbols()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    assert set(declared) == set(N.EXPORTED)
    assert lib.sq_version() >= 100
    assert lib.sq_error_string(N.SQ_ERR_SHAPE).decode()


def test_native_packed_layout_matches_reference_tables():
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.pool import packed_layout
    for entry in load_layouts():
        bits = torch.tensor(entry["bits"])
        plan = QuantizationPlan(entry["architecture"], bits, torch.ones_like(bits).float(), entry["value_group_size"])
        got = packed_layout(plan, entry["values"], entry["storage"])
        assert list(got) == [entry["offsets"], entry["rows"], entry["columns"], entry["page_bytes"]]


def test_layout_rejects_bad_storage_and_widths():
    from stepquant_b200 import _native as N
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.pool import packed_layout
    plan = QuantizationPlan("gdn", torch.full((1, 4), 6), torch.ones(1, 4))
    with pytest.raises(ValueError):
        packed_layout(plan, 8, "nibble")
    bits = (ctypes.c_int32 * 4)(6, 6, 7, 6)
    out = (ctypes.c_int32 * 8)()
    page = ctypes.c_int64()
    assert N.lib().sq_packed_layout(0, 1, 4, 8, 32, bits, 0, out, out, out, ctypes.byref(page)) == N.SQ_ERR_ARGUMENT
    # 3 and 5 bits are the width extension: the C layout takes them, a plan only with extended_widths.
    bits = (ctypes.c_int32 * 4)(5, 5, 5, 5)
    assert N.lib().sq_packed_layout(0, 1, 4, 8, 32, bits, 0, out, out, out, ctypes.byref(page)) == N.SQ_OK
    with pytest.raises(ValueError):
        QuantizationPlan("gdn", torch.full((1, 4), 5), torch.ones(1, 4))
    ext = QuantizationPlan("kda", torch.tensor([[3, 5, 16, 4]]), torch.ones(1, 4), extended_widths=True)
    from oracle import stepquant_oracle as O
    assert packed_layout(ext, 8) == O.packed_layout(O.Plan("kda", ext.bits.numpy(), ext.impact.numpy(),
                                                           extended_widths=True), 8)


def test_device_entry_points_reject_bad_arguments_before_launch():
    from stepquant_b200 import _native as N
    plan = N.SqPlan(0, 2, 128, 128, 32, 0, 1000, None, None, None, None, None)
    assert N.lib().sq_encode(ctypes.byref(plan), None, None, 1, None, 4, None, None) == N.SQ_ERR_ARGUMENT
    fake = ctypes.c_void_p(16)
    plan = N.SqPlan(0, 2, 96, 128, 32, 0, 1000, fake, fake, fake, fake, fake)
    assert N.lib().sq_decode(ctypes.byref(plan), fake, 4, fake, 1, fake, None, None) == N.SQ_ERR_SHAPE
    plan = N.SqPlan(0, 2, 128, 128, 2, 0, 1000, fake, fake, fake, fake, fake)
    assert N.lib().sq_decode(ctypes.byref(plan), fake, 4, fake, 1, fake, None, None) == N.SQ_ERR_UNSUPPORTED
    plan = N.SqPlan(0, 4, 128, 128, 32, 0, 1000, fake, fake, fake, fake, fake)
    args = N.SqStepArgs(16, 16, 16, 0, 0, 0, 3, 0, 16, 16, 0, 0, None, None, 1.0, 0, 16)
    assert N.lib().sq_step(ctypes.byref(plan), fake, 4, fake, 1, ctypes.byref(args), None, None, None) == N.SQ_ERR_SHAPE
    assert N.lib().sq_pack(fake, 4, 7, fake, None) == N.SQ_ERR_ARGUMENT
    # Page storage codes: 0 packed, 1 byte carriers, 2 / 3 baseline formats; others are rejected.
    for storage, code in ((4, N.SQ_ERR_ARGUMENT), (-1, N.SQ_ERR_ARGUMENT), (3, N.SQ_ERR_SHAPE)):
        plan = N.SqPlan(0, 2, 96, 128, 32, storage, 1000, fake, fake, fake, fake, fake)
        assert N.lib().sq_decode(ctypes.byref(plan), fake, 4, fake, 1, fake, None, None) == code
    assert N.lib().sq_packed_bytes(7, 6) == 6 and N.lib().sq_packed_bytes(0, 2) == 0
    # Zero-size work is a no-op that touches no pointer.
    assert N.lib().sq_pack(None, 0, 4, None, None) == N.SQ_OK


def test_quantization_plan_validation():
    from stepquant_b200 import QuantizationPlan
    with pytest.raises(ValueError):
        QuantizationPlan("mamba", torch.full((1, 4), 6), torch.ones(1, 4))
    with pytest.raises(ValueError):
        QuantizationPlan("gdn", torch.tensor([[4, 6, 4, 4]]), torch.ones(1, 4))
    with pytest.raises(ValueError):
        QuantizationPlan("kda", torch.tensor([[3, 6, 4, 4]]), torch.ones(1, 4))
    with pytest.raises(ValueError):
        QuantizationPlan("kda", torch.full((1, 4), 6), torch.zeros(1, 4))
    with pytest.raises(ValueError):
        QuantizationPlan("kda", torch.full((1, 4), 6), torch.ones(1, 4), value_group_size=0)
    QuantizationPlan("kda", torch.tensor([[2, 4, 8, 16]]), torch.ones(1, 4))


def test_cpu_tensors_fail_loudly():
    from stepquant_b200 import QuantizationPlan, fit_state
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.packing import pack
    plan = QuantizationPlan("gdn", torch.full((1, 4), 6), torch.ones(1, 4))
    with pytest.raises(ValueError):
        PackedStatePool(plan, 2, 8)
    with pytest.raises(ValueError):
        pack(torch.zeros(8, dtype=torch.int16), 4)
    with pytest.raises(ValueError):
        fit_state(torch.zeros(1, 1, 4, 8), plan)


def test_format_registry():
    from stepquant_b200.formats import BASELINE_NAMES, FORMAT_NAMES, get_format
    assert set(BASELINE_NAMES) == {"fp32", "sym_int4_g128", "sym_int6_g128", "sym_int8_g128", "dsq_int4", "dsq_int6"}
    assert get_format("stepquant6").bits == 6 and get_format("stepquant4").calibrated
    assert get_format("dsq_int4").group_axis == "k" and get_format("sym_int8_g128").group_size == 128
    assert FORMAT_NAMES[-2:] == ["stepquant4", "stepquant6"]
    for name in ("fp16", "bf16", "fp8", "dsq_int8", "sym_int4_g32"):
        with pytest.raises(ValueError, match="unknown state format"):
            get_format(name)


def test_profile_tiers_and_invalid_batches():
    from stepquant_b200.kernels.profiles import stepquant6_profile
    for arch in ("gdn", "kda"):
        for batch in (1, 17, 32, 33, 64, 65, 128, 129, 256, 257, 512):
            profile = stepquant6_profile(arch, batch)
            assert 0 < profile.sms <= 148 and profile.sms % 8 == 0
            assert profile.chunk % 32 == 0
        assert stepquant6_profile(arch, 33) == stepquant6_profile(arch, 64)
    for batch in (0, 513, True, 32.5):
        with pytest.raises(ValueError):
            stepquant6_profile("gdn", batch)
    with pytest.raises(ValueError):
        stepquant6_profile("unsupported", 32)


@pytest.mark.parametrize("chunk", [32, 64, 128, 256, 512])
def test_kda_release_keeps_forward_tail_bounded(monkeypatch, chunk):
    # test_writeback_schedule.py:9-23: the release schedule never accumulates
    # writeback work across recurrent layers.
    from stepquant_b200.kernels.writeback import CapturedWrites
    monkeypatch.setattr(torch.cuda, "Event", lambda **kwargs: SimpleNamespace(record=lambda: None))
    tasks = CapturedWrites(attention_windows=True)
    slots = torch.arange(512)
    recurrent = [True, True, True, False] * 6 + [True, True, False]
    chunks = (len(slots) + chunk - 1) // chunk
    for is_recurrent in recurrent:
        tasks.release_window()
        if is_recurrent:
            pool = SimpleNamespace(plan=SimpleNamespace(architecture="kda"), storage="packed",
                                   early_writeback=True, writeback_chunk=chunk)
            tasks.append((pool, slots))
        assert len(tasks.pending) <= chunks
    assert not tasks.pending
    assert len(tasks) == sum(recurrent) * chunks
    assert sum(task.final for task in tasks) == sum(recurrent)


def test_captured_writes_reject_double_layer_write(monkeypatch):
    from stepquant_b200.kernels.writeback import CapturedWrites
    monkeypatch.setattr(torch.cuda, "Event", lambda **kwargs: SimpleNamespace(record=lambda: None))
    tasks = CapturedWrites()
    pool = SimpleNamespace(plan=SimpleNamespace(architecture="gdn"), storage="packed", writeback_chunk=3)
    tasks.append((pool, torch.arange(7)))
    assert [len(t.tensors[0]) for t in tasks] + [len(p[1][0]) for p in tasks.pending] == [3, 3, 1] or len(tasks) + len(tasks.pending) == 3
    with pytest.raises(ValueError):
        tasks.append((pool, torch.arange(7)))


def test_prefill_arguments_are_checked_before_any_launch():
    """chunk_gated_delta_rule / chunk_kda reject bad shapes and CPU tensors on
    the host (ValueError / NotImplementedError), with no CPU fallback."""
    from stepquant_b200.kernels.prefill import chunk_gated_delta_rule, chunk_kda
    q = torch.randn(10, 2, 128, dtype=torch.bfloat16)
    v3 = torch.randn(10, 3, 128, dtype=torch.bfloat16)
    v2 = torch.randn(10, 2, 128, dtype=torch.bfloat16)
    beta = torch.rand(10, 2)
    for run in (chunk_gated_delta_rule, chunk_kda):
        with pytest.raises(ValueError):
            run(q, q, v3, beta, beta)  # 3 value heads over 2 qk heads
        small = torch.randn(10, 2, 64, dtype=torch.bfloat16)
        with pytest.raises(NotImplementedError):
            run(small, small, small, beta, beta)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(q, q, v2, beta, beta)  # CPU tensors
    with pytest.raises(ValueError):
        chunk_kda(q, q, v2, torch.zeros(10, 2, 128), beta)  # CPU tensors
