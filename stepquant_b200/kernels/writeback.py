"""Deferred background writeback under CUDA-graph capture.

Public names and behaviour follow stepquant/kernels/writeback.py
(``attention_window``, ``defer_writeback``, ``CapturedWrites``,
``WritebackChunk``, ``WritebackGraph``); the scheduler below is this
package's own.

While a forward pass is captured, each layer's requantization is queued as
*pieces* of at most ``writeback_chunk`` requests (0: the whole batch).  Queued
pieces leave the queue only at a *gate*: a point of the capture where one
event is recorded on the capturing stream and the next pieces are handed to
the writeback stream behind it, so they overlap whatever the forward does
after that point.  How many pieces a gate takes, and whether one opens right
after a layer's foreground step, is ``_gate_policy``:

* without attention windows every layer's pieces go out in two halves, one
  gate right after its foreground step and one at the start of the next
  layer's step, so the background never lags more than a layer behind;
* with attention windows (``attention_window()`` placed before attention
  work) a GDN layer releases everything at once, a KDA layer that writes back
  early releases at least half (and at least three) pieces per gate, and
  other KDA layers wait for the next window;
* the end of the capture opens one last gate for whatever is still queued.

In a *joined* capture released pieces are captured into the forward graph on
the writeback stream; in a *paired* capture they are recorded as
``WritebackChunk`` entries that ``WritebackGraph`` captures into a second,
background graph replayed on the writeback stream after the forward graph.
"""
from collections import deque
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass
from typing import NamedTuple

import torch

_active = ContextVar("stepquant_b200_writeback_capture", default=None)


@dataclass
class WritebackChunk:
    """A released piece: its pool, the gate event it waits for, its scratch views."""
    pool: object
    ready: torch.cuda.Event
    tensors: tuple
    final: bool  # the layer's last piece (its pool's graph_ready is recorded after it)


class _Piece(NamedTuple):
    pool: object
    tensors: tuple
    final: bool


def _split(pool, tensors):
    """The pieces of one layer's writeback, in request order."""
    batch = tensors[-1].numel()
    size = pool.writeback_chunk or batch or 1
    return [_Piece(pool, tuple(t[lo:min(lo + size, batch)] for t in tensors), lo + size >= batch)
            for lo in range(0, batch, size)]


def _gate_policy(pool, pieces, attention_windows):
    """(pieces a gate releases, whether a gate opens right after the layer's step)."""
    half = -(-pieces // 2)
    if not attention_windows:
        return half, True
    if pool.plan.architecture == "kda":
        if pool.storage == "byte" or getattr(pool, "early_writeback", False):
            return max(min(pieces, 3), half), True
        return pieces, False
    return pieces, True


def _enqueue(chunk):
    """Put one released piece on its pool's writeback stream behind its gate."""
    with torch.cuda.stream(chunk.pool.writeback_stream):
        chunk.ready.wait()
        chunk.pool._finish_update(*chunk.tensors)


class CapturedWrites(list):
    """The released pieces of one capture (list entries) plus the queue of
    pieces still waiting for a gate (``pending``)."""

    def __init__(self, attention_windows=False, joined=False):
        super().__init__()
        self.attention_windows = attention_windows
        self.joined = joined
        self.window_count = 0
        self.pending = deque()
        self.quota = 0
        self.layers = set()

    def release_window(self, count=None):
        """Open a gate for up to ``count`` queued pieces (default: the current quota)."""
        take = min(self.quota if count is None else count, len(self.pending))
        if take <= 0:
            return
        gate = torch.cuda.Event(external=not self.joined)
        gate.record()
        for _ in range(take):
            pool, tensors, final = self.pending.popleft()
            chunk = WritebackChunk(pool, gate, tensors, final)
            super().append(chunk)
            if self.joined:
                _enqueue(chunk)

    def append(self, task):
        """Queue a layer's writeback: ``(pool, *scratch tensors)``, slots last."""
        pool, *tensors = task
        if id(pool) in self.layers:
            raise ValueError("a layer may write its state only once per forward graph")
        self.layers.add(id(pool))
        pieces = _split(pool, tensors)
        self.pending.extend(pieces)
        self.quota, open_now = _gate_policy(pool, len(pieces), self.attention_windows)
        if open_now:
            self.release_window()


def attention_window():
    """Capture-time gate placed before attention work (counted when the capture uses windows)."""
    tasks = _active.get()
    if tasks is not None and tasks.attention_windows:
        tasks.window_count += 1
        tasks.release_window()


def _bind(pools, tasks):
    for pool in pools:
        pool.deferred = tasks


@contextmanager
def defer_writeback(pools, *, attention_windows=False, joined=False):
    """Collect the writeback of ``pools`` while a forward pass is captured.

    Yields the ``CapturedWrites`` of the capture.  On exit every queued piece is
    released; a joined capture also makes the capturing stream wait for the
    writeback stream, so the forward graph ends with every page written."""
    pools = tuple(pools)
    if any(pool.deferred is not None for pool in pools):
        raise RuntimeError("nested writeback capture is unsupported")
    tasks = CapturedWrites(attention_windows, joined)
    _bind(pools, tasks)
    token = _active.set(tasks)
    try:
        yield tasks
        if attention_windows and tasks.layers and not tasks.window_count:
            raise RuntimeError("no attention release hooks executed during graph capture")
    finally:
        _active.reset(token)
        tasks.release_window(len(tasks.pending))
        if joined and len(tasks):
            torch.cuda.current_stream().wait_stream(tasks[0].pool.writeback_stream)
        _bind(pools, None)


class WritebackGraph:
    """A captured forward graph and, for a paired capture, its background graph.

    ``replay()`` orders the forward after any earlier writeback of its pools,
    replays it, replays the background graph on the writeback stream (paired),
    and records one completion event that every pool then waits on."""

    def __init__(self, forward, tasks, joined=False):
        self.forward = forward
        self.tasks = tasks  # keeps the captured scratch views alive across replays
        self.pools = tuple(dict.fromkeys(chunk.pool for chunk in tasks))
        self.stream = tasks[0].pool.writeback_stream
        if any(pool.writeback_stream != self.stream for pool in self.pools):
            raise ValueError("captured layers must share one writeback stream")
        self.completion = torch.cuda.Event(external=True)
        self.background = None if joined else self._capture_background()

    def _capture_background(self):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self.stream):
            for chunk in self.tasks:
                chunk.ready.wait()
                chunk.pool._finish_update(*chunk.tensors)
                if chunk.final:
                    chunk.pool.graph_ready.record()
        for chunk in self.tasks:
            for tensor in chunk.tensors:
                tensor.record_stream(self.stream)
        return graph

    def replay(self):
        current = torch.cuda.current_stream()
        # Earlier writes of these pools (another graph, eager steps, slot
        # operations), each distinct completion event once.
        for event in dict.fromkeys(pool.completion for pool in self.pools if pool.pending):
            current.wait_event(event)
        self.forward.replay()
        if self.background is not None:
            with torch.cuda.stream(self.stream):
                self.background.replay()
                self.completion.record()
        else:
            # The joined forward graph already waits for its writes.
            self.completion.record(current)
            for pool in self.pools:
                if pool.captured_consumers:
                    pool.graph_ready.record(current)
        for pool in self.pools:
            pool.completion = self.completion
            pool.pending = True
