"""SGLang hook layer on the host (SGLang itself is not installed: fakes stand in,
as in the reference's own hook tests)."""
from types import SimpleNamespace

import pytest
import torch

from stepquant_b200.sglang import plugin, runtime


def test_writeback_settings_resolve_env(monkeypatch):
    from stepquant_b200.kernels.profiles import stepquant6_profile
    monkeypatch.setenv("STEPQUANT_STATE_FORMAT", "stepquant6")
    monkeypatch.setenv("STEPQUANT_WRITEBACK_SMS", "auto")
    monkeypatch.setenv("STEPQUANT_WRITEBACK_CHUNK", "auto")
    for arch, batch in (("gdn", 32), ("gdn", 512), ("kda", 512)):
        p = stepquant6_profile(arch, batch)
        assert runtime.writeback_settings(arch, batch) == (p.sms, p.chunk)
    monkeypatch.setenv("STEPQUANT_WRITEBACK_SMS", "0")
    assert runtime.writeback_settings("kda", 512) == (0, stepquant6_profile("kda", 512).chunk)
    monkeypatch.setenv("STEPQUANT_WRITEBACK_CHUNK", "0")
    assert runtime.writeback_settings("kda", 512) == (0, 0)
    monkeypatch.setenv("STEPQUANT_STATE_FORMAT", "stepquant4")
    monkeypatch.setenv("STEPQUANT_WRITEBACK_SMS", "56")
    monkeypatch.setenv("STEPQUANT_WRITEBACK_CHUNK", "256")
    assert runtime.writeback_settings("gdn", 32) == (56, 256)
    monkeypatch.delenv("STEPQUANT_WRITEBACK_SMS")
    monkeypatch.delenv("STEPQUANT_WRITEBACK_CHUNK")
    assert runtime.writeback_settings("gdn", 32) == (32, 64)


def _artifact(heads_total=8, keys=16, nominal=6):
    gen = torch.Generator().manual_seed(0)
    plans = {}
    for layer in (0, 3):
        bits = torch.tensor([4, 6, 6, 8] * (heads_total // 4))[:, None].expand(heads_total, keys).clone()
        plans[f"model.layers.{layer}.linear_attn"] = dict(
            architecture="gdn", bits=bits, impact=torch.rand(heads_total, keys, generator=gen) + 0.5,
            value_group_size=32)
    return dict(format_version=2, plans=plans, settings=dict(nominal_bits=nominal))


def test_local_plans_shard_value_heads(monkeypatch):
    art = _artifact()
    monkeypatch.setattr(runtime, "artifact", lambda: art)
    monkeypatch.setenv("STEPQUANT_STATE_FORMAT", "stepquant6")
    plans = [runtime.local_plans([3, 0], 2, "cpu", 16, rank=r, world=4) for r in range(4)]
    for layer_index, layer in ((0, 3), (1, 0)):
        full = art["plans"][f"model.layers.{layer}.linear_attn"]
        assert torch.equal(torch.cat([p[layer_index].bits for p in plans]), full["bits"])
        assert torch.equal(torch.cat([p[layer_index].impact for p in plans]), full["impact"])
    with pytest.raises(ValueError, match="head count"):
        runtime.local_plans([0], 3, "cpu", 16, rank=0, world=4)
    monkeypatch.setenv("STEPQUANT_STATE_FORMAT", "stepquant4")
    with pytest.raises(ValueError, match="nominal bits"):
        runtime.local_plans([0], 2, "cpu", 16, rank=0, world=4)


def test_server_arg_refusals():
    def server(**kw):
        base = dict(disable_radix_cache=True, enable_mamba_extra_buffer=lambda: False, pp_size=1,
                    enable_dp_attention=False, speculative_algorithm=None, disaggregation_mode="null",
                    linear_attn_backend="triton")
        base.update(kw)
        return SimpleNamespace(**base)
    runtime.check_server_args(server())
    for kw, match in ((dict(disable_radix_cache=False), "radix"), (dict(enable_mamba_extra_buffer=lambda: True), "no_buffer"),
                      (dict(pp_size=2), "tensor parallelism"), (dict(speculative_algorithm="eagle"), "speculative"),
                      (dict(disaggregation_mode="prefill"), "disaggregated"), (dict(linear_attn_backend="fla"), "triton")):
        with pytest.raises(ValueError, match=match):
            runtime.check_server_args(server(**kw))


def test_kernel_hooks_fall_through_for_other_pools():
    calls = []

    def original(self, *args, **kwargs):
        calls.append((args, kwargs))
        return "native"

    dense = torch.zeros(1)
    assert runtime.kernel_decode(original, None, 1, 2, 3, 4, 5, A_log=None, dt_bias=None, ssm_states=dense,
                                 cache_indices=None, query_start_loc=None) == "native"
    assert runtime.kernel_packed_decode(original, None, 1, 2, 3, A_log=None, dt_bias=None, scale=1., ssm_states=dense,
                                        cache_indices=None, num_v_heads=1, head_v_dim=1) == "native"
    assert runtime.kernel_extend(original, None, 1, 2, 3, 4, 5, ssm_states=dense, cache_indices=None,
                                 query_start_loc=None) == "native"
    assert len(calls) == 3


def test_temporal_pages_account_bytes():
    pages = runtime.TemporalPages([SimpleNamespace(nbytes=100), SimpleNamespace(nbytes=28)])
    assert pages.numel() == 128 and pages.shape == (128,) and pages.element_size() == 1
    with pytest.raises(NotImplementedError):
        pages[0:1]


def test_plugin_hook_targets_and_inactive_register(monkeypatch):
    targets = dict(plugin.hook_targets({"STEPQUANT_ASYNC_WRITEBACK": "1", "STEPQUANT_ARCHITECTURE": "gdn"}))
    assert targets["mem_cache.memory_pool.MambaPool.__init__"] == "pool_init"
    assert targets["layers.attention.linear.kernels.gdn_triton.TritonGDNKernel.packed_decode"] == "kernel_packed_decode"
    assert "model_executor.cuda_graph_runner.CudaGraphRunner.capture_one_batch_size" in targets
    assert all(hasattr(runtime, name) for name in targets.values())
    assert "model_executor.cuda_graph_runner.CudaGraphRunner.capture_one_batch_size" not in dict(plugin.hook_targets({}))
    monkeypatch.delenv("STEPQUANT_PLAN", raising=False)
    monkeypatch.delenv("STEPQUANT_STATE_FORMAT", raising=False)
    assert plugin.register() is None  # no settings: nothing imported, nothing registered


def test_page_bytes_per_slot_matches_layout(monkeypatch):
    from stepquant_b200 import QuantizationPlan
    from stepquant_b200.kernels.pool import packed_layout
    monkeypatch.setenv("STEPQUANT_STATE_FORMAT", "stepquant6")
    plans = [QuantizationPlan("gdn", torch.full((4, 128), b), torch.ones(4, 128)) for b in (4, 6, 8)]
    assert runtime.page_bytes_per_slot(plans, 128) == sum(packed_layout(p, 128)[-1] for p in plans)
