"""SGLang 0.5.12 hooks: packed Mamba pool, GDN/KDA dispatch and the writeback schedule.

Mirrors stepquant/sglang/runtime.py with this package's pool.  SGLang's model,
convolution cache, attention backend and scheduler stay native: the pool hooks
replace the dense recurrent cache by one ``PackedStatePool`` per layer, the
kernel hooks route decode (``kernel_decode`` / ``kernel_packed_decode``) and the
end of prefill (``kernel_extend``) through it, and ``capture_graph`` captures
the background writeback with ``defer_writeback`` / ``WritebackGraph``.

Settings come from the environment (as set by the reference's launcher):
STEPQUANT_PLAN, STEPQUANT_STATE_FORMAT, STEPQUANT_ARCHITECTURE,
STEPQUANT_ASYNC_WRITEBACK, STEPQUANT_WRITEBACK_SMS, STEPQUANT_WRITEBACK_CHUNK,
STEPQUANT_STATE_STORAGE.
"""
import dataclasses
import functools
import inspect
import logging
import os
import re
import weakref

import torch

from ..formats import FormatPlan, get_format
from ..kernels.format_pool import FormatStatePool, format_layout
from ..kernels.pool import PackedStatePool
from ..quantization import QuantizationPlan

log = logging.getLogger(__name__)
_temporal_pools = weakref.WeakSet()
_writeback_profiles = {}


@functools.lru_cache(maxsize=1)
def artifact():
    """The calibration plan file (torch.load, format_version 2)."""
    value = torch.load(os.environ["STEPQUANT_PLAN"], map_location="cpu", weights_only=True)
    if value.get("format_version") != 2:
        raise ValueError("unsupported STEPQuant plan format")
    return value


def state_format():
    return get_format(os.environ.get("STEPQUANT_STATE_FORMAT", "stepquant"))


def writeback_settings(architecture, batch):
    """Writeback (SMs, chunk) for a captured batch; 'auto' uses the STEPQuant@6 profile."""
    from ..kernels.profiles import stepquant6_profile
    nominal_six = state_format().name == "stepquant6"
    profile = stepquant6_profile(architecture, batch) if nominal_six else None
    sms = os.environ.get("STEPQUANT_WRITEBACK_SMS", "auto" if nominal_six else "32")
    chunk = os.environ.get("STEPQUANT_WRITEBACK_CHUNK", "auto" if nominal_six else "64")
    return (profile.sms if sms == "auto" else int(sms), profile.chunk if chunk == "auto" else int(chunk))


def tp_rank_world():
    """(rank, world) of SGLang's tensor-parallel group."""
    from sglang.srt.distributed import get_tensor_model_parallel_rank, get_tensor_model_parallel_world_size
    return get_tensor_model_parallel_rank(), get_tensor_model_parallel_world_size()


def shard_plan(entry, heads, rank, world, cls=QuantizationPlan):
    """This rank's value heads of a layer plan: bits/impact rows [rank*heads, (rank+1)*heads)."""
    plan = cls(**{k: v for k, v in entry.items() if k in ("architecture", "bits", "impact", "value_group_size")})
    if plan.bits.shape[0] != heads * world:
        raise ValueError("calibration head count does not match tensor-parallel shard")
    rows = slice(rank * heads, (rank + 1) * heads)
    return cls(plan.architecture, plan.bits[rows].contiguous(), plan.impact[rows].contiguous(), plan.value_group_size)


def local_plans(layer_ids, heads, device, keys=128, rank=None, world=None):
    """One plan per layer for this tensor-parallel rank (runtime.py:47-77)."""
    if rank is None or world is None:
        rank, world = tp_rank_world()
    spec = state_format()
    if not spec.calibrated:
        architecture = os.environ["STEPQUANT_ARCHITECTURE"]
        return [FormatPlan(architecture, torch.full((heads, keys), spec.bits, dtype=torch.long),
                           torch.ones(heads, keys)).to(device) for _ in layer_ids]
    expected = artifact().get("state_format", "stepquant")
    if spec.name in ("stepquant4", "stepquant6") and artifact().get("settings", {}).get("nominal_bits") != spec.bits:
        raise ValueError("plan nominal bits do not match the requested STEPQuant format")
    if expected != "stepquant":
        raise ValueError(f"{expected} plan requires its matching --state-format")
    mapping = {}
    for name, entry in artifact()["plans"].items():
        match = re.search(r"\.layers\.(\d+)\.", name)
        if not match:
            raise ValueError(f"cannot map layer name {name}")
        mapping[int(match[1])] = entry
    return [shard_plan(mapping[layer], heads, rank, world).to(device) for layer in layer_ids]


class TemporalPages:
    """Stands in for SGLang's dense temporal cache tensor: one pool per layer."""

    def __init__(self, pages):
        self.pages = pages
        _temporal_pools.add(self)

    def __getitem__(self, index):
        if not isinstance(index, int):
            raise NotImplementedError("use packed pool slot operations")
        return self.pages[index]

    def numel(self):
        return sum(p.nbytes for p in self.pages)

    def element_size(self):
        return 1

    @property
    def shape(self):
        return (self.numel(),)

    dtype = torch.uint8


def make_pool(plan, size, values, spec, stream, workspace, chunk, storage):
    if spec.kind == "stepquant":
        return PackedStatePool(plan, size + 1, values, writeback_stream=stream, writeback_workspace=workspace,
                               writeback_chunk=chunk, storage=storage)
    return FormatStatePool(plan, size + 1, values, spec, writeback_stream=stream)


def pool_init(original, self, **kwargs):
    if kwargs.get("speculative_num_draft_tokens") is not None:
        raise ValueError("STEPQuant currently does not support speculative decoding")
    params = kwargs["cache_params"]
    heads, values, keys = params.shape.temporal  # SGLang stores [H, V, K]
    plans = local_plans(kwargs["mamba_layer_ids"], heads, kwargs["device"], keys)
    if any(p.bits.shape[1] != keys for p in plans):
        raise ValueError("calibration key dimension mismatch")
    # SGLang initialises its convolution cache and allocators with an empty
    # temporal shape, so the dense recurrent pool is never allocated.
    tiny = dataclasses.replace(params, shape=dataclasses.replace(params.shape, temporal=(heads, 0, 0)))
    original(self, **dict(kwargs, cache_params=tiny))
    stream = None
    architecture = plans[0].architecture if plans else os.environ.get("STEPQUANT_ARCHITECTURE", "gdn")
    sms, chunk = writeback_settings(architecture, min(512, max(1, kwargs["size"])))
    if os.environ.get("STEPQUANT_ASYNC_WRITEBACK") == "1":
        from ..kernels.resources import writeback_resources
        resources = writeback_resources(kwargs["device"], sms)
        stream = resources.stream
        log.warning("STEPQuant background SMs: requested=%d actual=%d total=%d",
                    resources.requested_sms, resources.actual_sms, resources.total_sms)
        os.environ["STEPQUANT_WRITEBACK_ACTUAL_SMS"] = str(resources.actual_sms)
    spec = state_format()
    storage = os.environ.get("STEPQUANT_STATE_STORAGE", "packed")
    workspace = {}
    pages = TemporalPages([make_pool(p, kwargs["size"], values, spec, stream, workspace, chunk, storage) for p in plans])
    self.mamba_cache = dataclasses.replace(self.mamba_cache, temporal=pages)
    self.mem_usage = self.mamba_cache.mem_usage_bytes() / 1024 ** 3
    dense = len(plans) * (kwargs["size"] + 1) * heads * values * keys * 4
    log.warning("STEPQuant state pool (%s): %d bytes (FP32 %d bytes), %d layers, slots=%d",
                storage, pages.numel(), dense, len(plans), kwargs["size"] + 1)


def pool_alloc(original, self, need_size):
    if need_size > len(self.free_slots):
        return None
    slots = self.free_slots[:need_size]
    self.free_slots = self.free_slots[need_size:]
    for conv in self.mamba_cache.conv:
        conv[:, slots] = 0
    for p in self.mamba_cache.temporal.pages:
        p.clear(slots)
    return slots


def pool_copy_from(original, self, src_index, dst_index):
    for conv in self.mamba_cache.conv:
        conv[:, dst_index] = conv[:, src_index]
    for p in self.mamba_cache.temporal.pages:
        p.copy(src_index, dst_index)


def pool_get_cpu_copy(original, self, indices):
    """Raw page bytes of the given slots (the page layout is the wire format)."""
    torch.cuda.synchronize()
    return ([c[:, indices].cpu() for c in self.mamba_cache.conv],
            [p.data[indices].cpu() for p in self.mamba_cache.temporal.pages])


def pool_load_cpu_copy(original, self, mamba_cache_cpu, indices):
    convs, pages = mamba_cache_cpu
    for dst, src in zip(self.mamba_cache.conv, convs):
        dst[:, indices] = src.to(dst.device)
    for dst, src in zip(self.mamba_cache.temporal.pages, pages):
        dst.wait()
        dst.data[indices] = src.to(dst.device)


def pool_get_contiguous_buf_infos(original, self):
    raise NotImplementedError("STEPQuant does not support disaggregated serving")


def kernel_decode(original, self, q, k, v, a, b, *, A_log, dt_bias, ssm_states, cache_indices, query_start_loc,
                  **kwargs):
    if not isinstance(ssm_states, PackedStatePool):
        return original(self, q, k, v, a, b, A_log=A_log, dt_bias=dt_bias, ssm_states=ssm_states,
                        cache_indices=cache_indices, query_start_loc=query_start_loc, **kwargs)
    out = ssm_states.step(q, k, v, a, b, cache_indices, normalize=True, scale=ssm_states.keys ** -0.5,
                          a_log=A_log, dt_bias=dt_bias)
    return out.unsqueeze(0)


def kernel_packed_decode(original, self, mixed_qkv, a, b, *, A_log, dt_bias, scale, ssm_states, cache_indices,
                         num_v_heads, head_v_dim, **kwargs):
    if not isinstance(ssm_states, PackedStatePool):
        return original(self, mixed_qkv, a, b, A_log=A_log, dt_bias=dt_bias, scale=scale, ssm_states=ssm_states,
                        cache_indices=cache_indices, num_v_heads=num_v_heads, head_v_dim=head_v_dim, **kwargs)
    vdim = num_v_heads * head_v_dim
    kdim = (mixed_qkv.shape[-1] - vdim) // 2
    q, k, v = mixed_qkv.split([kdim, kdim, vdim], -1)
    return ssm_states.step(q, k, v, a, b, cache_indices, normalize=True, scale=scale, a_log=A_log,
                           dt_bias=dt_bias).unsqueeze(0)


def kernel_extend(original, self, q, k, v, g, beta, *, ssm_states, cache_indices, query_start_loc, **kwargs):
    """Prefill.  GDN pools with K = V = 128 run the chunked state pass of this
    library (``PackedStatePool.extend``: decode, chunk pass with in-kernel q/k
    L2 normalisation, encode).  Other packed pools decode the active pages, let
    the original chunk kernel update the dense V-first state in place, and
    encode the final state back into the pages (runtime.py:193-202)."""
    if not isinstance(ssm_states, PackedStatePool):
        return original(self, q, k, v, g, beta, ssm_states=ssm_states, cache_indices=cache_indices,
                        query_start_loc=query_start_loc, **kwargs)
    if ssm_states.plan.architecture == "gdn" and ssm_states.keys == 128 and ssm_states.values == 128:
        return ssm_states.extend(q, k, v, g, beta, cache_indices, query_start_loc, normalize=True)
    active = ssm_states.decode(cache_indices).transpose(-1, -2).contiguous()
    indices = torch.arange(cache_indices.numel(), device=cache_indices.device, dtype=cache_indices.dtype)
    output = original(self, q, k, v, g, beta, ssm_states=active, cache_indices=indices,
                      query_start_loc=query_start_loc, **kwargs)
    ssm_states.encode(active.transpose(-1, -2), cache_indices)
    return output


def attention_forward(original, self, *args, **kwargs):
    from ..kernels.writeback import attention_window
    attention_window()
    return original(self, *args, **kwargs)


def capture_graph(original, self, bs, forward, stream_idx=None):
    """Capture one decode batch size with deferred (joined) background writeback."""
    from ..kernels.writeback import WritebackGraph, defer_writeback
    if state_format().name == "stepquant6":
        from ..kernels.resources import writeback_resources
        pools = [pool for temporal in tuple(_temporal_pools) for pool in temporal.pages
                 if getattr(pool, "writeback_stream", None) is not None]
        resources = chunk = None
        for pool in pools:
            sms, chunk = writeback_settings(pool.plan.architecture, bs)
            resources = writeback_resources(pool.device, sms)
            pool.configure_writeback(resources.stream, chunk)
        if pools:
            _writeback_profiles[str(bs)] = dict(requested_sms=resources.requested_sms,
                                                actual_sms=resources.actual_sms, chunk=chunk)
            log.warning("STEPQuant6 capture: batch=%d background_sms=%d requested_sms=%d chunk=%d",
                        bs, resources.actual_sms, resources.requested_sms, chunk)
    tasks = []

    @functools.wraps(forward)
    def capture_forward(*args, **kwargs):
        if not torch.cuda.is_current_stream_capturing():
            return forward(*args, **kwargs)
        pools = [pool for temporal in tuple(_temporal_pools) for pool in temporal.pages
                 if getattr(pool, "writeback_stream", None) is not None]
        with defer_writeback(pools, attention_windows=True, joined=True) as captured:
            result = forward(*args, **kwargs)
        tasks.extend(captured)
        return result

    graph, output = original(self, bs, capture_forward, stream_idx)
    return (WritebackGraph(graph, tasks, joined=True) if tasks else graph), output


def validate_runner(original, self, *args, **kwargs):
    """Refuse server modes the packed pool does not support (runtime.py:271-294)."""
    from .plugin import verify_hooks
    verify_hooks()
    server = inspect.signature(original).bind(self, *args, **kwargs).arguments["server_args"]
    check_server_args(server)
    return original(self, *args, **kwargs)


def check_server_args(server):
    if not server.disable_radix_cache:
        raise ValueError("STEPQuant requires --disable-radix-cache until prefix-state tracking is enabled")
    if server.enable_mamba_extra_buffer():
        raise ValueError("STEPQuant requires --mamba-scheduler-strategy no_buffer")
    if getattr(server, "enable_memory_saver", False):
        raise ValueError("STEPQuant does not yet support SGLang memory-saver pause/resume")
    if getattr(server, "pp_size", 1) != 1 or getattr(server, "enable_dp_attention", False):
        raise ValueError("STEPQuant currently supports ordinary tensor parallelism only")
    if getattr(server, "speculative_algorithm", None):
        raise ValueError("STEPQuant does not support speculative decoding")
    if getattr(server, "disaggregation_mode", "null") not in ("null", None):
        raise ValueError("STEPQuant does not support disaggregated serving")
    if any(getattr(server, key, None) not in (None, "triton") for key in
           ("linear_attn_backend", "linear_attn_decode_backend", "linear_attn_prefill_backend")):
        raise ValueError("STEPQuant requires --linear-attn-backend triton")


def agree_min(count, group):
    """Smallest slot count over the ranks of ``group`` (a gloo CPU group); the
    mixed-precision page size differs per rank (runtime.py:310-317)."""
    if group is None or torch.distributed.get_world_size(group) <= 1:
        return count
    shared = torch.tensor(count, dtype=torch.int64)
    torch.distributed.all_reduce(shared, op=torch.distributed.ReduceOp.MIN, group=group)
    return int(shared.item())


def page_bytes_per_slot(plans, values, storage="packed"):
    """Bytes of one request slot over all layers' pools."""
    from ..kernels.pool import packed_layout
    spec = state_format()
    return sum((packed_layout(p, values, storage) if spec.kind == "stepquant" else format_layout(p, values, spec))[-1]
               for p in plans)


def size_pool(original, self, total_rest_memory):
    """Size SGLang's slot count by the packed page size instead of the dense state."""
    params = self.mambaish_config.mamba2_cache_params
    heads, values, keys = params.shape.temporal
    plans = local_plans(params.layers, heads, "cpu", keys)
    conv_bytes = sum(__import__("math").prod(shape) for shape in params.shape.conv) * params.dtype.conv.itemsize \
        * len(params.layers)
    compact = conv_bytes + page_bytes_per_slot(plans, values, os.environ.get("STEPQUANT_STATE_STORAGE", "packed"))
    dense = params.mamba_cache_per_req
    server = self.server_args
    if server.max_mamba_cache_size is None and not (server.disable_radix_cache and server.max_running_requests is not None):
        state_budget = total_rest_memory * server.mamba_full_memory_ratio / (1 + server.mamba_full_memory_ratio)
        count = max(0, int(state_budget * (1 << 30) // compact) - 1)
        from sglang.srt.distributed import get_tp_group
        group = get_tp_group()
        if group.world_size > 1:
            count = agree_min(count, group.cpu_group)
        if count < 1:
            raise ValueError("insufficient memory for a STEPQuant request slot")
        server.max_mamba_cache_size = count * (server.dp_size if server.enable_dp_attention else 1)
    result = original(self, total_rest_memory)
    # Upstream deducted the dense estimate; account for the packed bytes instead
    # (slot zero is the sentinel and is counted too).
    return result + (server.max_mamba_cache_size * (dense - compact) - compact) / (1 << 30)
