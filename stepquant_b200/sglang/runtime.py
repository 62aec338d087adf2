"""SGLang 0.5.12 hooks: packed state pools, GDN/KDA kernel routing, writeback schedule.

The hook names, their signatures (``original, self, ...``: AROUND hooks of
SGLang's HookRegistry), the SGLang attributes they touch and the environment
variables are those of stepquant/sglang/runtime.py, so the plugin is a drop-in;
the code below is organised around this package's pool.

* Settings: ``STEPQUANT_PLAN`` (calibration file), ``STEPQUANT_STATE_FORMAT``,
  ``STEPQUANT_ARCHITECTURE``, ``STEPQUANT_ASYNC_WRITEBACK``,
  ``STEPQUANT_WRITEBACK_SMS`` / ``_CHUNK`` and ``STEPQUANT_STATE_STORAGE``.
* Pools: SGLang's Mamba pool keeps its convolution cache and allocators; its
  dense recurrent ("temporal") cache is replaced by ``TemporalPages``, one
  ``PackedStatePool`` (or baseline-format pool) per layer with ``size + 1``
  slots (slot 0 is SGLang's padding sentinel).  Slot operations go to both.
* Kernels: decode routes to ``PackedStatePool.step``; prefill of GDN and KDA
  layers with K = V = 128 runs this package's state pass
  (``PackedStatePool.extend``), other layers let SGLang's chunk kernel update
  the decoded dense state in place.
* Graphs: each captured decode batch size defers its background writeback
  (``defer_writeback(..., attention_windows=True, joined=True)``) and the
  captured graph is returned wrapped in a ``WritebackGraph``.
"""
import dataclasses
import functools
import inspect
import logging
import math
import os
import re
import weakref

import torch

from ..formats import FormatPlan, get_format
from ..kernels.format_pool import FormatStatePool, format_layout
from ..kernels.pool import PackedStatePool
from ..quantization import QuantizationPlan

log = logging.getLogger(__name__)
_temporal_pools = weakref.WeakSet()   # every TemporalPages this process created
_writeback_profiles = {}              # captured batch size -> writeback SMs and chunk


# ---------------------------------------------------------------------------
# settings and the calibration file
# ---------------------------------------------------------------------------
def _env(name, default=None):
    return os.environ.get(name, default)


def state_format():
    return get_format(_env("STEPQUANT_STATE_FORMAT", "stepquant"))


def _storage():
    return _env("STEPQUANT_STATE_STORAGE", "packed")


@functools.lru_cache(maxsize=1)
def artifact():
    """The calibration plan file: ``torch.load(weights_only=True)``, format_version 2."""
    loaded = torch.load(_env("STEPQUANT_PLAN"), map_location="cpu", weights_only=True)
    if loaded.get("format_version") != 2:
        raise ValueError("unsupported STEPQuant plan format")
    return loaded


def writeback_settings(architecture, batch):
    """(writeback SMs, chunk) for ``batch``.  Under stepquant6 both default to
    'auto' (the ``stepquant6_profile`` tier of the batch), otherwise to 32 SMs
    and chunks of 64; the environment overrides either."""
    from ..kernels.profiles import stepquant6_profile
    tuned = state_format().name == "stepquant6"
    profile = stepquant6_profile(architecture, batch) if tuned else None
    resolved = []
    for var, field, fallback in (("STEPQUANT_WRITEBACK_SMS", "sms", "32"), ("STEPQUANT_WRITEBACK_CHUNK", "chunk", "64")):
        text = _env(var, "auto" if tuned else fallback)
        resolved.append(getattr(profile, field) if text == "auto" else int(text))
    return tuple(resolved)


def tp_rank_world():
    """(rank, world) of SGLang's tensor-parallel group."""
    from sglang.srt.distributed import get_tensor_model_parallel_rank, get_tensor_model_parallel_world_size
    return get_tensor_model_parallel_rank(), get_tensor_model_parallel_world_size()


def shard_plan(entry, heads, rank, world, cls=QuantizationPlan):
    """This rank's value heads of one layer's plan entry (rows rank*heads .. +heads)."""
    fields = ("architecture", "bits", "impact", "value_group_size")
    whole = cls(**{key: entry[key] for key in fields if key in entry})
    if whole.bits.shape[0] != heads * world:
        raise ValueError("calibration head count does not match tensor-parallel shard")
    lo, hi = rank * heads, (rank + 1) * heads
    return cls(whole.architecture, whole.bits[lo:hi].contiguous(), whole.impact[lo:hi].contiguous(),
               whole.value_group_size)


def _plans_by_layer(art):
    """Layer index -> plan entry, the index parsed from ``...layers.<i>....`` names."""
    table = {}
    for name, entry in art["plans"].items():
        found = re.search(r"\.layers\.(\d+)\.", name)
        if found is None:
            raise ValueError(f"cannot map layer name {name}")
        table[int(found.group(1))] = entry
    return table


def local_plans(layer_ids, heads, device, keys=128, rank=None, world=None):
    """One plan per layer in ``layer_ids`` for this tensor-parallel rank.

    Uncalibrated formats get a uniform plan of their width; calibrated ones are
    read from the plan file, which must carry the requested nominal width."""
    spec = state_format()
    if not spec.calibrated:
        width = torch.full((heads, keys), spec.bits, dtype=torch.long)
        return [FormatPlan(os.environ["STEPQUANT_ARCHITECTURE"], width, torch.ones(heads, keys)).to(device)
                for _ in layer_ids]
    art = artifact()
    if spec.name in ("stepquant4", "stepquant6") and art.get("settings", {}).get("nominal_bits") != spec.bits:
        raise ValueError("plan nominal bits do not match the requested STEPQuant format")
    saved = art.get("state_format", "stepquant")
    if saved != "stepquant":
        raise ValueError(f"{saved} plan requires its matching --state-format")
    if rank is None or world is None:
        rank, world = tp_rank_world()
    table = _plans_by_layer(art)
    return [shard_plan(table[layer], heads, rank, world).to(device) for layer in layer_ids]


# ---------------------------------------------------------------------------
# the pools standing in for SGLang's dense temporal cache
# ---------------------------------------------------------------------------
class TemporalPages:
    """SGLang's temporal cache tensor, replaced by one pool per layer.

    SGLang only indexes it by layer and asks for its byte size."""

    dtype = torch.uint8

    def __init__(self, pages):
        self.pages = pages
        _temporal_pools.add(self)

    def __getitem__(self, layer):
        if isinstance(layer, int):
            return self.pages[layer]
        raise NotImplementedError("use packed pool slot operations")

    def numel(self):
        return sum(pool.nbytes for pool in self.pages)

    def element_size(self):
        return 1

    @property
    def shape(self):
        return (self.numel(),)


def _async_pools():
    """Pools of every live TemporalPages that write back on a side stream."""
    return [pool for pages in tuple(_temporal_pools) for pool in pages.pages
            if getattr(pool, "writeback_stream", None) is not None]


def make_pool(plan, size, values, spec, stream, workspace, chunk, storage):
    if spec.kind != "stepquant":
        return FormatStatePool(plan, size + 1, values, spec, writeback_stream=stream)
    return PackedStatePool(plan, size + 1, values, writeback_stream=stream, writeback_workspace=workspace,
                           writeback_chunk=chunk, storage=storage)


def _writeback_stream(device, architecture, size):
    """(stream or None, chunk) for a pool of ``size`` requests."""
    sms, chunk = writeback_settings(architecture, min(512, max(1, size)))
    if _env("STEPQUANT_ASYNC_WRITEBACK") != "1":
        return None, chunk
    from ..kernels.resources import writeback_resources
    res = writeback_resources(device, sms)
    log.warning("STEPQuant background SMs: requested=%d actual=%d total=%d",
                res.requested_sms, res.actual_sms, res.total_sms)
    os.environ["STEPQUANT_WRITEBACK_ACTUAL_SMS"] = str(res.actual_sms)
    return res.stream, chunk


def pool_init(original, self, **kwargs):
    """MambaPool.__init__: SGLang builds everything but the dense temporal cache,
    which becomes one packed pool per recurrent layer."""
    if kwargs.get("speculative_num_draft_tokens") is not None:
        raise ValueError("STEPQuant currently does not support speculative decoding")
    params = kwargs["cache_params"]
    heads, values, keys = params.shape.temporal  # SGLang's order: [H, V, K]
    plans = local_plans(kwargs["mamba_layer_ids"], heads, kwargs["device"], keys)
    if any(plan.bits.shape[1] != keys for plan in plans):
        raise ValueError("calibration key dimension mismatch")
    empty = dataclasses.replace(params.shape, temporal=(heads, 0, 0))
    original(self, **{**kwargs, "cache_params": dataclasses.replace(params, shape=empty)})
    size = kwargs["size"]
    architecture = plans[0].architecture if plans else _env("STEPQUANT_ARCHITECTURE", "gdn")
    stream, chunk = _writeback_stream(kwargs["device"], architecture, size)
    spec, storage, workspace = state_format(), _storage(), {}
    pages = TemporalPages([make_pool(plan, size, values, spec, stream, workspace, chunk, storage) for plan in plans])
    self.mamba_cache = dataclasses.replace(self.mamba_cache, temporal=pages)
    self.mem_usage = self.mamba_cache.mem_usage_bytes() / 1024 ** 3
    log.warning("STEPQuant state pool (%s): %d bytes (FP32 %d bytes), %d layers, slots=%d", storage,
                pages.numel(), len(plans) * (size + 1) * heads * values * keys * 4, len(plans), size + 1)


def _each_cache(self, on_conv, on_pool):
    for conv in self.mamba_cache.conv:
        on_conv(conv)
    for pool in self.mamba_cache.temporal.pages:
        on_pool(pool)


def pool_alloc(original, self, need_size):
    """Take ``need_size`` free slots and zero their convolution and packed state."""
    if need_size > len(self.free_slots):
        return None
    slots, self.free_slots = self.free_slots[:need_size], self.free_slots[need_size:]

    def zero(conv):
        conv[:, slots] = 0
    _each_cache(self, zero, lambda pool: pool.clear(slots))
    return slots


def pool_copy_from(original, self, src_index, dst_index):
    def copy(conv):
        conv[:, dst_index] = conv[:, src_index]
    _each_cache(self, copy, lambda pool: pool.copy(src_index, dst_index))


def pool_get_cpu_copy(original, self, indices):
    """Host copies of the slots' convolution state and raw page bytes (the page
    layout is the wire format)."""
    torch.cuda.synchronize()
    convs, pages = [], []
    _each_cache(self, lambda conv: convs.append(conv[:, indices].cpu()),
                lambda pool: pages.append(pool.data[indices].cpu()))
    return convs, pages


def pool_load_cpu_copy(original, self, mamba_cache_cpu, indices):
    convs, pages = (iter(part) for part in mamba_cache_cpu)

    def load_conv(conv):
        conv[:, indices] = next(convs).to(conv.device)

    def load_pool(pool):
        pool.wait()
        pool.data[indices] = next(pages).to(pool.data.device)
    _each_cache(self, load_conv, load_pool)


def pool_get_contiguous_buf_infos(original, self):
    raise NotImplementedError("STEPQuant does not support disaggregated serving")


# ---------------------------------------------------------------------------
# kernels
# ---------------------------------------------------------------------------
def _packed(ssm_states):
    return isinstance(ssm_states, PackedStatePool)


def kernel_decode(original, self, q, k, v, a, b, *, A_log, dt_bias, ssm_states, cache_indices, query_start_loc,
                  **kwargs):
    """TritonGDNKernel / TritonKDAKernel.decode: one packed step, [1, B, H, V]."""
    if not _packed(ssm_states):
        return original(self, q, k, v, a, b, A_log=A_log, dt_bias=dt_bias, ssm_states=ssm_states,
                        cache_indices=cache_indices, query_start_loc=query_start_loc, **kwargs)
    return ssm_states.step(q, k, v, a, b, cache_indices, normalize=True, scale=ssm_states.keys ** -0.5,
                           a_log=A_log, dt_bias=dt_bias)[None]


def kernel_packed_decode(original, self, mixed_qkv, a, b, *, A_log, dt_bias, scale, ssm_states, cache_indices,
                         num_v_heads, head_v_dim, **kwargs):
    """TritonGDNKernel.packed_decode: q, k, v arrive concatenated in ``mixed_qkv``."""
    if not _packed(ssm_states):
        return original(self, mixed_qkv, a, b, A_log=A_log, dt_bias=dt_bias, scale=scale, ssm_states=ssm_states,
                        cache_indices=cache_indices, num_v_heads=num_v_heads, head_v_dim=head_v_dim, **kwargs)
    value_width = num_v_heads * head_v_dim
    key_width = (mixed_qkv.shape[-1] - value_width) // 2
    q, k, v = mixed_qkv.split([key_width, key_width, value_width], -1)
    return ssm_states.step(q, k, v, a, b, cache_indices, normalize=True, scale=scale, a_log=A_log,
                           dt_bias=dt_bias)[None]


def kernel_extend(original, self, q, k, v, g, beta, *, ssm_states, cache_indices, query_start_loc, **kwargs):
    """Prefill.  Pools with K = V = 128 run this package's state pass
    (``PackedStatePool.extend``: decode, the GDN chunk pass or the KDA
    recurrent pass with in-kernel q/k L2 normalisation, encode); g is the
    kernel's log decay as the layer hands it over ([.., T, H] for GDN,
    [.., T, H, K] for KDA).  Other packed pools hand SGLang's chunk kernel the
    decoded states, V-first as it keeps them, with the active requests
    numbered 0..n-1, and encode what it leaves there."""
    if not _packed(ssm_states):
        return original(self, q, k, v, g, beta, ssm_states=ssm_states, cache_indices=cache_indices,
                        query_start_loc=query_start_loc, **kwargs)
    if ssm_states.keys == 128 and ssm_states.values == 128:
        return ssm_states.extend(q, k, v, g, beta, cache_indices, query_start_loc, normalize=True)
    dense = ssm_states.decode(cache_indices).transpose(-1, -2).contiguous()
    local = torch.arange(cache_indices.numel(), device=cache_indices.device, dtype=cache_indices.dtype)
    out = original(self, q, k, v, g, beta, ssm_states=dense, cache_indices=local, query_start_loc=query_start_loc,
                   **kwargs)
    ssm_states.encode(dense.transpose(-1, -2), cache_indices)
    return out


def attention_forward(original, self, *args, **kwargs):
    """Decoder-layer forward: a writeback release gate before its attention work."""
    from ..kernels.writeback import attention_window
    attention_window()
    return original(self, *args, **kwargs)


# ---------------------------------------------------------------------------
# CUDA-graph capture
# ---------------------------------------------------------------------------
def _bind_capture_resources(bs):
    """stepquant6: give every async pool the writeback stream and chunk of the batch's profile tier."""
    from ..kernels.resources import writeback_resources
    chosen = None
    for pool in _async_pools():
        sms, chunk = writeback_settings(pool.plan.architecture, bs)
        res = writeback_resources(pool.device, sms)
        pool.configure_writeback(res.stream, chunk)
        chosen = (res, chunk)
    if chosen is not None:
        res, chunk = chosen
        _writeback_profiles[str(bs)] = dict(requested_sms=res.requested_sms, actual_sms=res.actual_sms, chunk=chunk)
        log.warning("STEPQuant6 capture: batch=%d background_sms=%d requested_sms=%d chunk=%d",
                    bs, res.actual_sms, res.requested_sms, chunk)


class _DeferredForward:
    """The forward SGLang captures, with the async pools' writeback deferred
    into the same graph (joined); eager calls pass straight through."""

    def __init__(self, forward):
        self.forward = forward
        self.chunks = []
        functools.update_wrapper(self, forward)

    def __call__(self, *args, **kwargs):
        if not torch.cuda.is_current_stream_capturing():
            return self.forward(*args, **kwargs)
        from ..kernels.writeback import defer_writeback
        with defer_writeback(_async_pools(), attention_windows=True, joined=True) as captured:
            result = self.forward(*args, **kwargs)
        self.chunks.extend(captured)
        return result


def capture_graph(original, self, bs, forward, stream_idx=None):
    """CudaGraphRunner.capture_one_batch_size: the graph, wrapped in a joined
    ``WritebackGraph`` when it captured writeback."""
    from ..kernels.writeback import WritebackGraph
    if state_format().name == "stepquant6":
        _bind_capture_resources(bs)
    deferred = _DeferredForward(forward)
    graph, output = original(self, bs, deferred, stream_idx)
    return (WritebackGraph(graph, deferred.chunks, joined=True) if deferred.chunks else graph), output


# ---------------------------------------------------------------------------
# server checks and pool sizing
# ---------------------------------------------------------------------------
_SERVER_RULES = (
    (lambda s: not s.disable_radix_cache,
     "STEPQuant requires --disable-radix-cache until prefix-state tracking is enabled"),
    (lambda s: s.enable_mamba_extra_buffer(), "STEPQuant requires --mamba-scheduler-strategy no_buffer"),
    (lambda s: getattr(s, "enable_memory_saver", False),
     "STEPQuant does not yet support SGLang memory-saver pause/resume"),
    (lambda s: getattr(s, "pp_size", 1) != 1 or getattr(s, "enable_dp_attention", False),
     "STEPQuant currently supports ordinary tensor parallelism only"),
    (lambda s: getattr(s, "speculative_algorithm", None), "STEPQuant does not support speculative decoding"),
    (lambda s: getattr(s, "disaggregation_mode", "null") not in ("null", None),
     "STEPQuant does not support disaggregated serving"),
    (lambda s: any(getattr(s, key, None) not in (None, "triton") for key in
                   ("linear_attn_backend", "linear_attn_decode_backend", "linear_attn_prefill_backend")),
     "STEPQuant requires --linear-attn-backend triton"),
)


def check_server_args(server):
    """Raise ValueError for the first server mode the packed pool cannot serve."""
    for refuses, message in _SERVER_RULES:
        if refuses(server):
            raise ValueError(message)


def validate_runner(original, self, *args, **kwargs):
    """ModelRunner.__init__: every hook installed, the server mode supported."""
    from .plugin import verify_hooks
    verify_hooks()
    check_server_args(inspect.signature(original).bind(self, *args, **kwargs).arguments["server_args"])
    return original(self, *args, **kwargs)


def agree_min(count, group):
    """Smallest slot count over the ranks of ``group`` (a CPU group): mixed
    precision gives ranks different page sizes, but every rank must offer the
    scheduler the same number of slots."""
    if group is None or torch.distributed.get_world_size(group) <= 1:
        return count
    shared = torch.tensor(count, dtype=torch.int64)
    torch.distributed.all_reduce(shared, op=torch.distributed.ReduceOp.MIN, group=group)
    return int(shared.item())


def page_bytes_per_slot(plans, values, storage="packed"):
    """Bytes of one request slot over all layers' pools."""
    from ..kernels.pool import packed_layout
    spec = state_format()
    if spec.kind == "stepquant":
        return sum(packed_layout(plan, values, storage)[-1] for plan in plans)
    return sum(format_layout(plan, values, spec)[-1] for plan in plans)


def size_pool(original, self, total_rest_memory):
    """ModelRunnerKVCacheMixin.handle_max_mamba_cache: size the slot count by the
    packed bytes of a request instead of SGLang's dense estimate, and return
    the memory SGLang deducted for dense slots that the packed pool leaves free."""
    params = self.mambaish_config.mamba2_cache_params
    heads, values, keys = params.shape.temporal
    conv = sum(math.prod(shape) for shape in params.shape.conv) * params.dtype.conv.itemsize * len(params.layers)
    slot_bytes = conv + page_bytes_per_slot(local_plans(params.layers, heads, "cpu", keys), values, _storage())
    server = self.server_args
    if server.max_mamba_cache_size is None and not (server.disable_radix_cache and
                                                    server.max_running_requests is not None):
        ratio = server.mamba_full_memory_ratio
        count = max(0, int(total_rest_memory * ratio / (1 + ratio) * (1 << 30) // slot_bytes) - 1)
        from sglang.srt.distributed import get_tp_group
        group = get_tp_group()
        if group.world_size > 1:
            count = agree_min(count, group.cpu_group)
        if count < 1:
            raise ValueError("insufficient memory for a STEPQuant request slot")
        server.max_mamba_cache_size = count * (server.dp_size if server.enable_dp_attention else 1)
    result = original(self, total_rest_memory)
    # The sentinel slot 0 is allocated too, so it is deducted once more.
    return result + (server.max_mamba_cache_size * (params.mamba_cache_per_req - slot_bytes) - slot_bytes) / (1 << 30)
