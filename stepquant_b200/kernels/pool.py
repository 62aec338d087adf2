"""Fixed-layout GPU pages, shared plan tables and request-slot operations.

``PackedStatePool`` is the drop-in for the reference's pool
(stepquant/kernels/pool.py:69-365): same constructor, attributes, page byte
layout (``packed_layout``) and stream/event semantics.  The arithmetic runs
in libstepquant_b200 (include/stepquant_b200.h):

* no writeback stream: ``step`` is one fused kernel (``sq_step``) that reads
  each page once and writes it once;
* with a writeback stream: ``sq_readout`` on the caller's stream produces the
  output, and ``sq_writeback`` requantizes on the writeback stream, immediately
  or deferred under graph capture (``writeback.defer_writeback``).  Both modes
  write identical page bytes.
"""
import ctypes

import torch

from .. import _native as N
from ..quantization import DevicePlan


def _capture_id(stream):
    from cuda.bindings import runtime
    status, _, identifier, *_ = runtime.cudaStreamGetCaptureInfo(stream.cuda_stream)
    if status != runtime.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cannot query CUDA capture: {status}")
    return identifier


def packed_layout(plan, value_dim, storage="packed"):
    """Page byte layout (kernels/pool.py:19-66): (offsets, rows, columns, page_bytes).

    offsets: code/pivot byte offset of each key row followed by each head's
    stride between value tiles; rows: fp16 row-scale offsets (-1 = pivot);
    columns: fp16 column-scale offsets (-1 = all-pivot head).
    """
    if storage not in ("packed", "byte"):
        raise ValueError("state storage must be packed or byte")
    bits = plan.bits.detach().to("cpu", torch.int32).contiguous()
    heads, keys = bits.shape
    offsets = (ctypes.c_int32 * (heads * keys + heads))()
    rows = (ctypes.c_int32 * (heads * keys))()
    columns = (ctypes.c_int32 * heads)()
    page = ctypes.c_int64()
    code = N.lib().sq_packed_layout(N.SQ_KDA if plan.architecture == "kda" else N.SQ_GDN, heads, keys, value_dim,
                                    plan.value_group_size, ctypes.c_void_p(bits.data_ptr()),
                                    1 if storage == "byte" else 0, offsets, rows, columns, ctypes.byref(page))
    N.check(code)
    return list(offsets), list(rows), list(columns), page.value


class PackedStatePool:
    def __init__(self, plan, slots, value_dim=128, writeback_stream=None, writeback_workspace=None,
                 writeback_chunk=64, storage="packed"):
        if plan.bits.device.type != "cuda":
            raise ValueError("state pool requires CUDA")
        if storage not in ("packed", "byte"):
            raise ValueError("state storage must be packed or byte")
        self.storage = storage
        self.early_writeback = True
        self.plan = plan
        self.heads, self.keys = plan.bits.shape
        self.values = value_dim
        if self.keys & (self.keys - 1) or value_dim & (value_dim - 1) or value_dim % 4:
            raise ValueError("key/value dimensions must be powers of two, value_dim >= 4")
        if plan.architecture == "gdn" and value_dim % plan.value_group_size:
            raise ValueError("value dimension must be divisible by value_group_size")
        if not 4 <= self.keys <= 128 or value_dim > 128:
            raise NotImplementedError("this build supports key and value dimensions from 4 to 128")
        self.device = plan.bits.device
        self._dp = DevicePlan(plan, value_dim, storage)
        self.page_bytes = self._dp.page_bytes
        self.offsets, self.rows, self.columns = self._dp.offsets, self._dp.rows, self._dp.columns
        self.bits, self.impact = self._dp.bits, self._dp.impact
        # Pages plus 64 bytes of tail padding for wide loads near the last page.
        self._storage = torch.zeros(slots * self.page_bytes + 64, device=self.device, dtype=torch.uint8)
        self.data = self._storage[:slots * self.page_bytes].view(slots, self.page_bytes)
        self.status = torch.zeros(1, device=self.device, dtype=torch.int32)
        self.coefficients = None
        self.row_tile = 0
        self._init_writeback(writeback_stream, writeback_chunk)
        self._init_workspace(slots, writeback_workspace)

    # -- writeback state ------------------------------------------------------
    # ready: recorded on the writeback stream after an eager writeback;
    # graph_ready: an external event every producer (eager or captured)
    # records, the one a consumer captured into another graph can wait on;
    # completion: the event the next consumer waits for (ready, graph_ready or
    # a WritebackGraph's completion); ready_capture: the capture that recorded
    # ready, if any.
    def _init_writeback(self, writeback_stream, writeback_chunk):
        if writeback_chunk < 0:
            raise ValueError("writeback chunk must be nonnegative")
        self.writeback_stream = writeback_stream
        self.writeback_chunk = writeback_chunk
        self.deferred = None
        self.pending = self.captured_consumers = False
        self.consumer_dependencies = set()
        self.ready_capture = None
        asynchronous = writeback_stream is not None
        self.ready = torch.cuda.Event() if asynchronous else None
        self.graph_ready = torch.cuda.Event(external=True) if asynchronous else None
        self.completion = self.ready
        if asynchronous:
            self.graph_ready.record(torch.cuda.current_stream(self.device))

    def _init_workspace(self, slots, writeback_workspace):
        self.scratch = None
        if self.writeback_stream is None:
            return
        # Writer inputs live outside any CUDA graph's private pool: a graph may
        # reuse a freed temporary for a later tensor and the next replay could
        # overwrite it before a deferred writeback reads it (pool.py:141-143).
        floats = int(N.lib().sq_scratch_floats(self._dp.ref()))
        self.scratch = (torch.empty((slots, floats), device=self.device, dtype=torch.float32),
                        torch.empty(slots, device=self.device, dtype=torch.int64))
        for tensor in self.scratch:
            tensor.record_stream(self.writeback_stream)
        self.writeback_workspace = writeback_workspace

    @property
    def nbytes(self):
        return self.data.numel()

    def configure_writeback(self, stream, chunk):
        """Bind a capture's writer without replacing state or scratch storage (pool.py:164-179)."""
        if self.writeback_stream is None or chunk < 0:
            raise ValueError("configuring writeback requires an asynchronous pool and nonnegative chunk")
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("select writeback resources before CUDA graph capture")
        self.wait()
        if stream != self.writeback_stream:
            for tensor in self.scratch:
                tensor.record_stream(stream)
            self.writeback_stream = stream
        self.writeback_chunk = chunk

    def check_status(self):
        """Raise if a kernel skipped a request whose slot index was outside the pool (synchronizes)."""
        value = int(self.status.item())
        if value & N.SQ_STATUS_SLOT_RANGE:
            self.status.zero_()
            raise IndexError("a request slot index was outside the state pool; that request was skipped")

    # -- page operations -------------------------------------------------------
    def encode(self, state, slots):
        self.wait()
        if state.shape != (slots.numel(), self.heads, self.keys, self.values):
            raise ValueError("state must be [active slots, heads, key, value]")
        if slots.numel():
            state = state.float().contiguous()
            slots = self._slots(slots)
            N.check(N.lib().sq_encode(self._dp.ref(), N.ptr(state), N.ptr(slots), slots.numel(), N.ptr(self.data),
                                      self.data.shape[0], N.ptr(self.status), N.stream_handle()))

    def decode(self, slots):
        self.wait()
        state = torch.empty((slots.numel(), self.heads, self.keys, self.values), device=self.device,
                            dtype=torch.float32)
        if slots.numel():
            slots = self._slots(slots)
            N.check(N.lib().sq_decode(self._dp.ref(), N.ptr(self.data), self.data.shape[0], N.ptr(slots),
                                      slots.numel(), N.ptr(state), N.ptr(self.status), N.stream_handle()))
        return state

    def extend(self, q, k, v, g, beta, slots, query_start_loc, *, normalize=True, scale=None):
        """Prefill ``slots``: decode their states, run the prefill pass over
        each request's tokens (request i owns tokens query_start_loc[i] ..
        query_start_loc[i + 1]) and encode the final states back -- the
        decode -> chunk kernel -> encode sequence of the reference hook
        (stepquant/sglang/runtime.py:193-202).  g is the log decay (GDN: per
        token and value head; KDA: per token, value head and key channel) and
        beta the activated gate, per token and value head.  Returns the
        outputs shaped like ``v`` (bf16)."""
        from .prefill import chunk_gated_delta_rule, chunk_kda
        active = self.decode(slots)
        run = chunk_kda if self.plan.architecture == "kda" else chunk_gated_delta_rule
        out, final = run(q, k, v, g, beta, scale=scale, initial_state=active, use_qk_l2norm_in_kernel=normalize,
                         cu_seqlens=query_start_loc)
        self.encode(final, slots)
        return out

    def _slots(self, slots):
        if slots.device != self.device or slots.dtype != torch.int64 or not slots.is_contiguous():
            slots = slots.to(device=self.device, dtype=torch.int64).contiguous()
        return slots

    def _step_args(self, q, k, v, g, beta, batch, normalize, scale, a_log, dt_bias, out):
        if g.dtype != beta.dtype:
            beta = beta.to(g.dtype)
        if a_log is not None:
            if dt_bias is None:
                raise ValueError("raw gates need both a_log and dt_bias")
            a_log = a_log.float().contiguous()
            dt_bias = dt_bias.float().contiguous()
        keep = (q, k, v, g, beta, a_log, dt_bias, out)
        args = N.SqStepArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), k.stride(0), v.stride(0),
                            q.shape[1], N.dtype_code(q.dtype), g.data_ptr(), beta.data_ptr(), N.dtype_code(g.dtype),
                            int(bool(normalize)), None if a_log is None else a_log.data_ptr(),
                            None if dt_bias is None else dt_bias.data_ptr(), float(scale), 0, out.data_ptr())
        return args, keep

    def step(self, q, k, v, g, beta, slots, *, normalize=False, scale=1., a_log=None, dt_bias=None,
             state_out=None):
        """One decode step for ``slots`` (pool.py:200-282); returns out [B, H, V] in q.dtype.

        ``state_out`` (optional fp32 [B, H, K, V]) receives the updated state
        before requantization (synchronous pools only).
        """
        self.wait()
        if self.deferred is not None and not self.deferred.attention_windows:
            self.deferred.release_window()
        batch = slots.numel()
        if not batch:
            return torch.empty((0, self.heads, self.values), device=q.device, dtype=q.dtype)
        q = q.reshape(batch, -1, self.keys)
        k = k.reshape(batch, -1, self.keys)
        v = v.reshape(batch, self.heads, self.values)
        if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
            raise ValueError("head coordinates must be contiguous")
        if q.stride(1) != self.keys or k.stride(1) != self.keys or v.stride(1) != self.values:
            raise ValueError("heads of one request must be contiguous")
        hq = q.shape[1]
        if self.heads % hq or k.shape[1] != hq:
            raise ValueError("value heads must be divisible by query heads")
        if k.dtype != q.dtype:
            k = k.to(q.dtype)
        if v.dtype != q.dtype:
            v = v.to(q.dtype)
        N.require_cuda(q, k, v, g, beta)
        g, beta = g.contiguous(), beta.contiguous()
        slots = self._slots(slots)
        out = torch.empty((batch, self.heads, self.values), device=q.device, dtype=q.dtype)
        args, keep = self._step_args(q, k, v, g, beta, batch, normalize, scale, a_log, dt_bias, out)
        if self.writeback_stream is not None:
            if batch > self.scratch[0].shape[0]:
                raise ValueError("active batch exceeds the state pool workspace capacity")
            scratch, stable = (t[:batch] for t in self.scratch)
            N.check(N.lib().sq_readout(self._dp.ref(), N.ptr(self.data), self.data.shape[0], N.ptr(slots), batch,
                                       ctypes.byref(args), N.ptr(scratch), N.ptr(stable), N.ptr(self.status),
                                       N.stream_handle()))
            self._schedule_writeback(scratch, stable)
        else:
            if state_out is not None and state_out.shape != (batch, self.heads, self.keys, self.values):
                raise ValueError("state_out must be [batch, heads, key, value] fp32")
            N.check(N.lib().sq_step(self._dp.ref(), N.ptr(self.data), self.data.shape[0], N.ptr(slots), batch,
                                    ctypes.byref(args), N.ptr(state_out), N.ptr(self.status), N.stream_handle()))
        del keep
        return out

    def _schedule_writeback(self, scratch, stable_slots):
        """Requantize on the writeback stream now, or queue it in the active deferral."""
        if self.deferred is not None:
            self.deferred.append((self, scratch, stable_slots))
            return
        producer = torch.cuda.current_stream(self.device)
        writer = self.writeback_stream
        writer.wait_stream(producer)
        with torch.cuda.stream(writer):
            self._finish_update(scratch, stable_slots)
            self.graph_ready.record(writer)
            self.ready.record(writer)
        scratch.record_stream(writer)
        stable_slots.record_stream(writer)
        capture = _capture_id(producer) if torch.cuda.is_current_stream_capturing() else None
        self.ready_capture = capture
        self.completion = self.ready if capture is None else self.graph_ready
        self.pending = True

    def _finish_update(self, scratch, stable_slots):
        """Requantize and repack the pages of one chunk on the current stream (pool.py:299-316)."""
        batch = stable_slots.numel()
        if not batch:
            return
        N.check(N.lib().sq_writeback(self._dp.ref(), N.ptr(self.data), self.data.shape[0], N.ptr(stable_slots),
                                     batch, N.ptr(scratch), None, N.ptr(self.status),
                                     N.stream_handle()))

    def _pending_events(self, stream):
        """The events ``stream`` must wait on before touching the pages."""
        if self.deferred is not None:  # inside a capture that defers this pool's writes
            return () if self.deferred.joined else (self.graph_ready,)
        if not self.pending:
            return ()
        if not torch.cuda.is_current_stream_capturing():
            return (self.completion,)
        if self.ready_capture == _capture_id(stream):
            return (self.ready,)  # produced earlier in this same capture
        # A consumer captured into a graph of its own: it waits on graph_ready,
        # which every later producer records too.  An event of an earlier
        # producer graph is kept alive, since graph nodes do not own events.
        self.captured_consumers = True
        if self.completion is self.ready or self.completion is self.graph_ready:
            return (self.graph_ready,)
        self.consumer_dependencies.add(self.completion)
        return (self.completion, self.graph_ready)

    def wait(self):
        """Order the current stream after pending writeback (reference pool.py:334-356)."""
        stream = torch.cuda.current_stream(self.device)
        for event in self._pending_events(stream):
            stream.wait_event(event)

    def clear(self, slots):
        self.wait()
        self.data[slots] = 0

    def copy(self, source, destination):
        self.wait()
        # Advanced indexing creates a temporary: an overlapping copy is well defined.
        self.data[destination] = self.data[source]
