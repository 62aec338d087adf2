#!/usr/bin/env python
"""Packed-state GDN decode benchmark on 1..8 B200s.

One *step* is one decode step of one GDN layer over the whole batch: for every
(request, value head) the packed state page is unpacked, the gated delta rule
applied, o = S^T q read out, the state requantized (fit_state), repacked and
written back.  Asynchronous writeback is on (config 1): the readout kernel runs
on the compute stream and the requantization on a writeback stream, and a
step is complete when both are.  ``--mode sync`` times the fused single-kernel
step instead.  The timed loop replays one CUDA graph per step (async steps
with their writeback joined; the end-to-end leg pairs a foreground graph with
a background writeback graph), as the
reference benchmark times ``step(); wait()`` under CUDA graphs; per-kernel
device times come from graph-captured batches of one kernel's launches timed
with CUDA events on that kernel's stream.

Workload: Qwen-Next-style layer, 16 qk heads / 32 value heads, K = V = 128,
batch 256, stepquant6 synthetic plan (seed 1: per-head widths {4, 6, 8} at
25/50/25, impact factors from a 256-step fp32 warm-up).  Value heads (and their
qk heads) are sharded over ranks as tensor parallelism does; no collective runs
in the timed state path.  Requests rotate over 4 groups of slots (a 420 MB pool
per GPU at N = 1, larger than the 126 MB L2), so each step reads pages that are
not L2-resident.

Other workloads: ``--workload kda-decode`` (config 2), ``gdn-prefill``
(config 3: chunked prefill to the first packed state), ``kda-prefill`` (the
same for KDA layers, recurrent fp32 pass) and ``gdn-stack``
(config 4: 48 GDN layers decoding through one CUDA graph per token, value heads
tensor-parallel with an NCCL all-gather of each layer's readout).

Prints one JSON line on rank 0.  ``--impl reference`` times the reference's CPU
path (StateCodec.decode -> delta_step -> StateCodec.encode, restated in numpy
by the oracle) on the host cores instead.
"""
import argparse
import contextlib
import ctypes
import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "packed-state decode updates/s"
_result_out = None


def emit(line):
    out = _result_out or sys.__stdout__
    out.write(json.dumps(line) + "\n")
    out.flush()
UNIT = "updates/s"


def parse_args():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("stepquant_b200", "reference", "reference-gpu"), default="stepquant_b200",
                   help="reference: the CPU port of the reference path; reference-gpu: the reference's own "
                        "Triton/Gluon pool from baseline/_ref beside this library's, config 1, one GPU")
    p.add_argument("--mode", choices=("async", "sync"), default="async")
    p.add_argument("--workload", choices=("gdn-decode", "kda-decode", "gdn-prefill", "kda-prefill", "gdn-stack"),
                   default="gdn-decode",
                   help="config 1 (default), config 2, config 3 or config 4")
    p.add_argument("--kda-widths", default="2,4,6",
                   help="KDA row widths at 30/50/20 (kda-decode): 2,4,6 is the reference-legal twin of config 2's "
                        "3,4,6, which needs the 3/5-bit width extension")
    p.add_argument("--batch", type=int, default=0,
                   help="default: 256 (config 1), 512 (config 2), 32 (config 3), 512 (config 4)")
    p.add_argument("--tokens", type=int, default=2048, help="prompt length (gdn-prefill)")
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--qk-heads", type=int, default=0, help="default: heads / 2 (GDN), heads (KDA)")
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--pivot-heads", type=int, default=1,
                   help="GDN heads stored as fp16 pivots (1% of 32 heads rounds to 0; at least one exercises the fp16 path)")
    p.add_argument("--two-bit-heads", type=int, default=0,
                   help="GDN heads stored at 2 bits with value-group row scales (a stepquant4-style plan; 0 in config 1)")
    p.add_argument("--slot-groups", type=int, default=4)
    p.add_argument("--warm-steps", type=int, default=256)
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-secondary", action="store_true", help="skip the short config-2 / config-3 measurements")
    p.add_argument("--layers", type=int, default=48, help="GDN layers of the stack (gdn-stack, config 4)")
    p.add_argument("--hidden", type=int, default=5120, help="hidden size of the stack's projections (gdn-stack)")
    p.add_argument("--prompt", type=int, default=128, help="prompt tokens per request before decoding (gdn-stack)")
    p.add_argument("--writeback-chunk", type=int, default=0,
                   help="requests per writeback launch (gdn-stack); default: the stepquant6 profile's chunk")
    p.add_argument("--writeback-sms", type=int, default=0,
                   help="SM budget of the writeback stream's green context (gdn-stack); 0 (default): an ordinary "
                        "stream; -1: the stepquant6 profile's budget")
    return p.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def _clock_worker(index, conn):
    """Child process: poll NVML every millisecond until told to stop; send the samples back."""
    import time as _time
    samples = []
    try:
        import pynvml
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(index)
        max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
        conn.send("ready")
        while not conn.poll(0.001):
            samples.append((_time.time(), pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM),
                            pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)))
    except Exception:  # NVML unavailable: report no samples
        max_mhz = None
        conn.send("ready")
        conn.recv()
    conn.send((max_mhz, samples))


class ClockSampler:
    """SM clock and throttle reasons sampled every 1 ms by a separate process.

    Only samples taken between start() and stop() (the timed region) are kept.
    """

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        import multiprocessing as mp
        ctx = mp.get_context("spawn")
        self.conn, child = ctx.Pipe()
        self.proc = ctx.Process(target=_clock_worker, args=(index, child), daemon=True)
        self.proc.start()
        self.conn.recv()  # NVML initialised
        self.window = None
        self.max_mhz, self.samples = None, []

    def start(self):
        self.t0 = time.time()

    def stop(self):
        self.window = (self.t0, time.time())
        self.conn.send("stop")
        self.max_mhz, samples = self.conn.recv()
        self.proc.join(timeout=10)
        lo, hi = self.window
        self.samples = [(m, r) for t, m, r in samples if lo <= t <= hi]

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted(name for name, bit in self.REASONS.items() if any(r & bit for _, r in self.samples))
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


def measured_peak(key="hbm_gbs"):
    """(peak, source) from MEASURED_PEAKS.json, else the pool's earlier measurement."""
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            data = json.load(fh)
        if key in data:
            return float(data[key]), "measured"
    return fallback[key], "fallback"


def algorithmic_bytes(pool_page_bytes, heads_local, qk_local, batch, dim, kda=False):
    """Bytes one decode step must move (per rank): pages read+written, bf16 q/k/v in, gates, bf16 out."""
    pages = 2 * pool_page_bytes * batch
    inputs = batch * (2 * qk_local * dim + heads_local * dim) * 2
    gates = batch * heads_local * (dim * 4 + 4 if kda else 8)
    output = batch * heads_local * dim * 2
    return pages, inputs + gates + output


# ---------------------------------------------------------------------------
# CPU reference arm / baseline (oracle port of the reference's torch path)
# ---------------------------------------------------------------------------

_cpu_state = {}


def _cpu_init(seed, heads, qk_heads, dim, counts, counter, barrier):
    """Worker set-up: this worker's share of the batch (``counts[i]`` requests
    for the i-th worker to start)."""
    import numpy as np
    from oracle import stepquant_oracle as O
    with counter.get_lock():
        index = counter.value
        counter.value += 1
    requests = counts[index]
    _cpu_state["barrier"] = barrier
    rng = np.random.default_rng(seed)
    widths = np.array(([4] * (heads // 4) + [6] * (heads - 2 * (heads // 4)) + [8] * (heads // 4)))
    rng.shuffle(widths)
    bits = np.repeat(widths[:, None], dim, 1)
    plan = O.Plan("gdn", bits, (rng.random((heads, dim)) + 0.5).astype(np.float32))
    rng = np.random.default_rng(seed + 1000 + index)
    state = (rng.standard_normal((requests, heads, dim, dim)) * 0.1).astype(np.float32)
    packed = O.codec_encode(state, plan)
    q = rng.standard_normal((requests, qk_heads, dim)).astype(np.float32)
    k = rng.standard_normal((requests, qk_heads, dim)).astype(np.float32)
    v = rng.standard_normal((requests, heads, dim)).astype(np.float32)
    a = rng.standard_normal((requests, heads)).astype(np.float32)
    b = rng.standard_normal((requests, heads)).astype(np.float32)
    a_log = (rng.random(heads) * math.log(16)).astype(np.float32)
    _cpu_state.update(plan=plan, packed=packed, inputs=(q, k, v, a, b, a_log, np.zeros(heads, np.float32)), dim=dim)


def _cpu_step(_):
    """One reference decode step for this worker's requests: decode -> delta_step -> encode."""
    from oracle import stepquant_oracle as O
    s = _cpu_state
    q, k, v, a, b, a_log, dt_bias = s["inputs"]
    if q.shape[0]:
        plan = s["plan"]
        state = O.codec_decode(s["packed"], plan)
        qp, kp, g, beta = O.prepare_inputs(q, k, a, b, plan.bits.shape[0], kda=False, normalize=True,
                                           scale=s["dim"] ** -0.5, a_log=a_log, dt_bias=dt_bias)
        _, updated = O.delta_step(state, qp, kp, v, g, beta)
        s["packed"] = O.codec_encode(updated, plan)
    # Every worker takes exactly one task per step: none returns before all have finished theirs.
    s["barrier"].wait(timeout=600)
    return int(q.shape[0])


def cpu_reference(args, heads, qk_heads, batch, steps, warmup, budget_seconds=None):
    """Time the CPU port of the reference path on the host cores: each step is
    the whole batch, its requests split over one spawned worker per core.
    Stops early (after at least one timed step) once ``budget_seconds`` of
    timed steps have run.  Returns a dict."""
    import multiprocessing as mp
    cores = max(1, min(os.cpu_count() or 1, batch))
    counts = [batch // cores + (1 if i < batch % cores else 0) for i in range(cores)]
    ctx = mp.get_context("spawn")
    # One thread per worker process (the workers already use every core).
    for var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = "1"
    initargs = (args.seed, heads, qk_heads, args.dim, counts, ctx.Value("i", 0), ctx.Barrier(cores))
    with ctx.Pool(cores, initializer=_cpu_init, initargs=initargs) as pool:
        for _ in range(warmup):
            pool.map(_cpu_step, range(cores), chunksize=1)
        times, done = [], 0
        for _ in range(steps):
            t0 = time.perf_counter()
            done = sum(pool.map(_cpu_step, range(cores), chunksize=1))
            times.append(time.perf_counter() - t0)
            if budget_seconds is not None and sum(times) > budget_seconds:
                break
    per_step = sum(times) / len(times)
    return {"value": done * heads / per_step, "unit": UNIT, "cores": cores, "kind": "port",
            "steps": len(times), "ms_per_step": per_step * 1e3, "requests": done,
            "sample": f"{len(times)} full steps of {done} requests x {heads} heads (K=V={args.dim}) on {cores} "
                      f"worker processes, mean step {per_step * 1e3:.0f} ms"}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # The reference arm runs config 1 (the default workload's shapes), whole steps.
    batch = args.batch or 256
    qk_heads = args.qk_heads or args.heads // 2
    res = cpu_reference(args, args.heads, qk_heads, batch, args.steps, args.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "gdn-decode-b%d-h%d-k128 (config 1), CPU port of the reference torch path"
                                   % (batch, args.heads),
                       "batch": batch, "heads": args.heads, "qk_heads": qk_heads, "dim": args.dim},
            "cpu_baseline": res, "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}
    emit(line)


def reference_gpu_arm(args):
    """The reference's own GPU path beside this library's on one B200.

    The unmodified reference package, installed into ``baseline/_ref`` (pip
    ``--target``; it is not part of this repository), runs config 1 through its
    public ``PackedStatePool`` (Triton/Gluon kernels, asynchronous writeback),
    timed the way its ``benchmarks/bench_formats.py`` times it: ``step();
    wait()`` captured in a CUDA graph (one per slot group and input set) and
    replayed between CUDA events.  This library's pool runs the identical plan,
    states, inputs and graph structure in the same process.  After encoding and
    after one step from the same pages the two pools' bytes and outputs are
    compared.  Rank 0 only; prints one JSON line.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = os.path.join(ROOT, "baseline", "_ref")
    base = {"impl": "reference-gpu", "metric": METRIC, "unit": UNIT}
    if not os.path.isdir(os.path.join(path, "stepquant")):
        emit(dict(base, unavailable="the reference package is not installed in baseline/_ref"))
        return
    import torch
    sys.path.insert(0, path)
    try:
        from stepquant.kernels.pool import PackedStatePool as RefPool
        from stepquant.quantization import QuantizationPlan as RefPlan
    except Exception as exc:  # an import failure of the reference is its result here
        emit(dict(base, unavailable="reference import failed: %s: %s" % (type(exc).__name__, exc)))
        return
    from stepquant_b200 import synthetic as S
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.quantization import QuantizationPlan

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    kda = args.workload == "kda-decode"
    arch = "kda" if kda else "gdn"
    batch, heads, dim = args.batch or (512 if kda else 256), args.heads, args.dim
    qk = args.qk_heads or (heads if kda else heads // 2)
    groups_n = 2 if kda else args.slot_groups
    cpu_gen = torch.Generator().manual_seed(2 if kda else args.seed)
    if kda:  # config 2's reference-legal twin plan: row widths {2,4,6} at 30/50/20, 2 % fp16 pivot rows
        bits = S.kda_widths(heads, dim, cpu_gen, choices=(2, 4, 6))
        plan_desc = "row widths {2,4,6} 30/50/20, 2% fp16 pivot rows, impact uniform [0.5, 1.5)"
    else:
        widths = S.gdn_widths(heads, cpu_gen, args.pivot_heads, args.two_bit_heads)
        bits = widths[:, None].expand(heads, dim).contiguous()
        plan_desc = ("widths {4,6,8} 25/50/25, pivot heads %d, 2-bit heads %d, impact uniform [0.5, 1.5)"
                     % (args.pivot_heads, args.two_bit_heads))
    impact = torch.rand(heads, dim, generator=cpu_gen) + 0.5
    gen = torch.Generator(device=device).manual_seed(args.seed)
    a_log, dt_bias = S.gate_parameters(heads, dim, kda, gen, device)
    kw = dict(normalize=True, scale=dim ** -0.5, a_log=a_log, dt_bias=dt_bias)
    slots_total = batch * groups_n + 1
    groups = [torch.arange(1 + g * batch, 1 + (g + 1) * batch, device=device) for g in range(groups_n)]
    inputs = [S.draw_inputs(batch, heads, qk, dim, dim, kda, gen, device) for _ in range(2)]
    state = torch.randn(batch * groups_n, heads, dim, dim, generator=gen, device=device) * 0.1

    def make(kind, asynchronous=True):
        stream = torch.cuda.Stream(device) if asynchronous else None
        if kind == "reference":
            return RefPool(RefPlan(arch, bits.to(device), impact.to(device)), slots_total, dim,
                           writeback_stream=stream)
        return PackedStatePool(QuantizationPlan(arch, bits.to(device), impact.to(device)), slots_total, dim,
                               writeback_stream=stream)

    def run(pool, i):
        x = inputs[i % len(inputs)]
        out = pool.step(x.q, x.k, x.v, x.a, x.b, groups[i % groups_n], **kw)
        pool.wait()
        return out

    def timed(pool, clocks=None):
        for i in range(args.warmup):
            run(pool, i)
        torch.cuda.synchronize()
        period = math.lcm(len(inputs), groups_n)
        graphs = []
        for j in range(period):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                run(pool, j)
            graphs.append(graph)
        for i in range(args.warmup):
            graphs[i % period].replay()
        torch.cuda.synchronize()
        start, end = _events()
        if clocks:
            clocks.start()
        start.record()
        for i in range(args.steps):
            graphs[i % period].replay()
        end.record()
        torch.cuda.synchronize()
        if clocks:
            clocks.stop()
        # Device time per step by kernel (torch profiler over one replay of each graph).
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for graph in graphs:
                graph.replay()
            torch.cuda.synchronize()
        kernels = {}
        for ev in prof.key_averages():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                kernels[ev.key[:60]] = kernels.get(ev.key[:60], 0.0) + ev.device_time_total / period
        del graphs
        return start.elapsed_time(end) / args.steps, {k: round(v, 1) for k, v in sorted(kernels.items(), key=lambda kv: -kv[1])}

    ours, theirs = make("this"), make("reference")
    for pool in (ours, theirs):
        pool.encode(state, torch.arange(1, slots_total, device=device))
    torch.cuda.synchronize()
    del state
    # One step from the same pages: compare the pools' bytes and outputs.
    same_layout = ours.data.shape == theirs.data.shape
    enc_equal = float((ours.data == theirs.data).float().mean()) if same_layout else None
    out_ours, out_theirs = run(ours, 0), run(theirs, 0)
    torch.cuda.synchronize()
    rows = groups[0]
    step_equal = float((ours.data[rows] == theirs.data[rows]).float().mean()) if same_layout else None
    out_diff = float((out_ours.float() - out_theirs.float()).abs().max())
    # The parity step advanced group 0 in both pools alike; the timed runs continue from there.
    clocks = ClockSampler(0)
    try:
        ref_ms, ref_kernels = timed(theirs, clocks)
    except Exception as exc:
        emit(dict(base, unavailable="reference step failed: %s: %s" % (type(exc).__name__, exc)))
        return
    our_ms, our_kernels = timed(ours)
    page_bytes, page_bytes_ours = theirs.page_bytes, ours.page_bytes
    del ours, theirs
    # The same comparison without a writeback stream (the fused / synchronous step of each).
    sync = {}
    for kind in ("reference", "this"):
        pool = make(kind, asynchronous=False)
        pool.encode(torch.randn(batch * groups_n, heads, dim, dim, generator=gen, device=device) * 0.1,
                    torch.arange(1, slots_total, device=device))
        ms, kernels = timed(pool)
        sync[kind] = {"ms_per_step": ms, "kernel_us_per_step": kernels}
        del pool
    updates = batch * heads
    import triton
    line = dict(base, value=updates / (ref_ms / 1e3), n_gpus=1, steps=args.steps, warmup=args.warmup,
                ms_per_step=ref_ms, higher_is_better=True, scaling="strong", vs_baseline=None, dtype="f32",
                data="synthetic",
                config={"workload": "%s-decode-b%d-h%d-k128 (config %d), reference Triton/Gluon PackedStatePool"
                                    % (arch, batch, heads, 2 if kda else 1), "batch": batch, "heads": heads,
                        "qk_heads": qk, "dim": dim, "plan": plan_desc,
                        "writeback": "async (reference default chunk 64)",
                        "timing": "step(); wait() in one CUDA graph per step, CUDA events",
                        "l2": "slots rotate over %d groups (%.0f MB of pages)"
                              % (groups_n, slots_total * page_bytes / 1e6)},
                triton=triton.__version__, clocks=clocks.summary(),
                kernel_us_per_step=ref_kernels,
                this_build={"value": updates / (our_ms / 1e3), "ms_per_step": our_ms,
                            "speedup_over_reference": ref_ms / our_ms, "kernel_us_per_step": our_kernels},
                synchronous={"reference_ms_per_step": sync["reference"]["ms_per_step"],
                             "this_build_ms_per_step": sync["this"]["ms_per_step"],
                             "speedup_over_reference": sync["reference"]["ms_per_step"] / sync["this"]["ms_per_step"],
                             "reference_kernel_us_per_step": sync["reference"]["kernel_us_per_step"],
                             "this_build_kernel_us_per_step": sync["this"]["kernel_us_per_step"]},
                parity={"page_bytes_equal_after_encode": enc_equal, "page_bytes_equal_after_step": step_equal,
                        "out_max_abs_diff": out_diff, "page_bytes": page_bytes,
                        "page_bytes_this_build": page_bytes_ours})
    emit(line)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def _events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def kernel_times(pool, inputs, groups, kw, mode, launches=8, reps=4):
    """Average device time (ms) of one launch of each decode kernel.

    ``launches`` launches of one kernel (rotating over the slot groups, so the
    pages they read exceed L2 as in the timed loop) are captured in a CUDA
    graph and replayed ``reps`` times between CUDA events on the stream the
    kernel runs on.  Launch-issue time on the host is thus kept out of the
    figure at every GPU count.
    """
    import torch
    from stepquant_b200 import _native as N

    batch = groups[0].numel()
    inp = inputs[0]
    out = torch.empty(batch, pool.heads, pool.values, device=inp.q.device, dtype=inp.q.dtype)
    args, keep = pool._step_args(inp.q, inp.k, inp.v, inp.a, inp.b, batch, kw["normalize"], kw["scale"], kw["a_log"],
                                 kw["dt_bias"], out)
    lib = N.lib()

    def readout(g):
        scratch, stable = (t[:batch] for t in pool.scratch)
        N.check(lib.sq_readout(pool._dp.ref(), N.ptr(pool.data), pool.data.shape[0], N.ptr(groups[g]), batch,
                               ctypes.byref(args), N.ptr(scratch), N.ptr(stable), N.ptr(pool.status),
                               N.stream_handle()))

    def writeback(g):
        # the readout's scratch of group 0, applied to group g's pages
        N.check(lib.sq_writeback(pool._dp.ref(), N.ptr(pool.data), pool.data.shape[0], N.ptr(groups[g]), batch,
                                 N.ptr(pool.scratch[0]), None, N.ptr(pool.status), N.stream_handle()))

    def step(g):
        N.check(lib.sq_step(pool._dp.ref(), N.ptr(pool.data), pool.data.shape[0], N.ptr(groups[g]), batch,
                            ctypes.byref(args), None, N.ptr(pool.status), N.stream_handle()))

    def timed(launch, stream):
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for j in range(launches):
                launch(j % len(groups))
        with torch.cuda.stream(stream):
            graph.replay()
            e0, e1 = _events()
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (reps * launches)

    pool.wait()
    compute = torch.cuda.Stream(inp.q.device)
    if mode != "async":
        result = {"step": timed(step, compute)}
    else:
        result = {"readout": timed(readout, compute)}
        readout(0)  # the writeback's inputs
        torch.cuda.synchronize()
        result["writeback"] = timed(writeback, torch.cuda.Stream(inp.q.device))
    del keep
    return result


def measure_decode(args, kda, batch, heads_total, qk_total, steps, warmup, world, rank, device, barrier,
                   mode="async", e2e=True, clocks=None, warm_steps=256, slot_groups=4, seed=1, kda_widths=(2, 4, 6)):
    """Decode steps of one layer (GDN config 1 or KDA config 2); returns the measured quantities."""
    import torch
    from stepquant_b200 import _native as N
    from stepquant_b200 import synthetic as S
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.writeback import WritebackGraph, defer_writeback
    from stepquant_b200.quantization import QuantizationPlan

    dim = args.dim
    heads_l, qk_l = heads_total // world, qk_total // world
    gen = torch.Generator(device=device).manual_seed(seed * 1000 + rank)
    cpu_gen = torch.Generator().manual_seed(seed)
    if kda:
        bits = S.kda_widths(heads_total, dim, cpu_gen, choices=tuple(kda_widths))[rank * heads_l:(rank + 1) * heads_l]
    else:
        widths = S.gdn_widths(heads_total, cpu_gen, args.pivot_heads, args.two_bit_heads)[rank * heads_l:(rank + 1) * heads_l]
        bits = widths[:, None].expand(heads_l, dim).clone()
    a_log, dt_bias = S.gate_parameters(heads_l, dim, kda, gen, device)
    requests = batch * slot_groups
    slots_total = requests + 1

    # fp32 warm-up state (the FP32 pool kernel) and row-impact statistics.
    fp32 = torch.zeros(slots_total, heads_l, dim, dim, device=device)
    warm_slots = torch.arange(1, slots_total, device=device)
    out_scratch = torch.empty(requests, heads_l, dim, device=device, dtype=torch.bfloat16)
    omega = torch.zeros(heads_l, dim, device=device, dtype=torch.float64)
    for _ in range(warm_steps):
        inp = S.draw_inputs(requests, heads_l, qk_l, dim, dim, kda, gen, device)
        st = N.SqStepArgs(inp.q.data_ptr(), inp.k.data_ptr(), inp.v.data_ptr(), inp.q.stride(0), inp.k.stride(0),
                          inp.v.stride(0), qk_l, N.SQ_BF16, inp.a.data_ptr(), inp.b.data_ptr(), N.SQ_F32, 1,
                          a_log.data_ptr(), dt_bias.data_ptr(), dim ** -0.5, 0, out_scratch.data_ptr())
        N.check(N.lib().sq_fp32_step(N.ptr(fp32), slots_total, heads_l, dim, dim, 1 if kda else 0, N.ptr(warm_slots),
                                     requests, ctypes.byref(st), None, N.stream_handle()))
        q, k, g, beta = S.prepared(inp, heads_l, dim, kda, a_log, dt_bias)
        omega += S.row_impact(q, k, g, beta).double().sum(0)
    impact = S.impact_factors(omega / (warm_steps * requests))
    extended = bool(kda and any(w in (3, 5) for w in kda_widths))  # the 3/5-bit width extension
    plan = QuantizationPlan("kda" if kda else "gdn", bits.to(device), impact.to(device), extended_widths=extended)

    stream = torch.cuda.Stream(device) if mode == "async" else None
    # One writeback launch per step (no chunking), as the eager path does.
    pool = PackedStatePool(plan, slots_total, dim, writeback_stream=stream, writeback_chunk=0)
    pool.encode(fp32[1:], warm_slots)
    del fp32
    groups = [torch.arange(1 + g * batch, 1 + (g + 1) * batch, device=device) for g in range(slot_groups)]
    inputs = [S.draw_inputs(batch, heads_l, qk_l, dim, dim, kda, gen, device) for _ in range(4)]
    kw = dict(normalize=True, scale=dim ** -0.5, a_log=a_log, dt_bias=dt_bias)

    def one_step(i):
        inp = inputs[i % len(inputs)]
        return pool.step(inp.q, inp.k, inp.v, inp.a, inp.b, groups[i % len(groups)], **kw)

    for i in range(warmup):
        one_step(i)
    pool.wait()
    barrier()
    kernel_ms = kernel_times(pool, inputs, groups, kw, mode)

    # The timed loop replays one CUDA graph per (inputs, slot group) pair -- the
    # reference benchmark's methodology (bench_formats.py times step(); wait()
    # under CUDA graphs).  Async steps are captured with their writeback
    # (defer_writeback + WritebackGraph): joined into one graph for the device
    # throughput; for the end-to-end leg as a foreground graph plus a
    # background writeback graph on the writeback stream (paired), so the next
    # step's host-to-device input copy overlaps the previous step's writeback.
    period = math.lcm(len(inputs), len(groups))

    def capture(step_fn, joined):
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        if mode != "async":
            with torch.cuda.graph(graph):
                result = step_fn()
            return graph, result
        with torch.cuda.graph(graph):
            with defer_writeback([pool], joined=joined) as tasks:
                result = step_fn()
        return WritebackGraph(graph, tasks, joined=joined), result

    graphs = [capture(lambda j=j: pool.step(inputs[j % len(inputs)].q, inputs[j % len(inputs)].k,
                                           inputs[j % len(inputs)].v, inputs[j % len(inputs)].a,
                                           inputs[j % len(inputs)].b, groups[j % len(groups)], **kw),
                      joined=True)[0]
              for j in range(period)]
    for i in range(warmup):
        graphs[i % period].replay()
    pool.wait()
    barrier()
    start, end = _events()
    barrier()
    if clocks:
        clocks.start()
    start.record()
    for i in range(steps):
        graphs[i % period].replay()
    pool.wait()
    end.record()
    barrier()
    if clocks:
        clocks.stop()
    res = {"elapsed_ms": start.elapsed_time(end), "kernel_ms": kernel_ms}
    del graphs
    pool.check_status()
    res["page_bytes"] = pool.page_bytes
    res["pivot_heads_local"] = 0 if kda else int((bits[:, 0] == 16).sum())
    res["two_bit_heads_local"] = 0 if kda else int((bits[:, 0] == 2).sum())
    res["algorithmic"] = algorithmic_bytes(pool.page_bytes, heads_l, qk_l, batch, dim, kda)

    if e2e:
        # Each step's inputs (q, k, v bf16; gates fp32) packed in one pinned host
        # buffer and copied with one H2D transfer; the output comes back with one D2H.
        fields = [(x.shape, x.dtype) for x in (inputs[0].q, inputs[0].k, inputs[0].v, inputs[0].a, inputs[0].b)]
        sizes = [math.prod(sh) * torch.tensor([], dtype=dt).element_size() for sh, dt in fields]
        offsets = [0]
        for nbytes in sizes:
            offsets.append(offsets[-1] + (nbytes + 255) // 256 * 256)
        pinned = []
        for x in inputs:
            buf = torch.empty(offsets[-1], dtype=torch.uint8).pin_memory()
            for t, o, nbytes in zip((x.q, x.k, x.v, x.a, x.b), offsets, sizes):
                buf[o:o + nbytes].copy_(t.contiguous().view(-1).view(torch.uint8).cpu())
            pinned.append(buf)
        # Two input buffers.  Each step is one captured graph (writeback joined):
        # on a copy stream it brings step i + 1's inputs from pinned host memory
        # into the other buffer while the step runs, and on another it copies the
        # step's output back to pinned host memory -- a serving loop's pipeline,
        # with the host issuing one graph launch per step.
        nbuf = 2
        dev_bufs = [torch.empty(offsets[-1], dtype=torch.uint8, device=device) for _ in range(nbuf)]
        dev_ins = [tuple(buf[o:o + nbytes].view(dt).view(sh) for (sh, dt), o, nbytes in zip(fields, offsets, sizes))
                   for buf in dev_bufs]
        host_outs = [torch.empty(batch, heads_l, dim, dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
        h2d, d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        e2e_period = math.lcm(period, nbuf)

        def e2e_graph(i):
            b, nb = i % nbuf, (i + 1) % nbuf
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                main = torch.cuda.current_stream()
                deferral = defer_writeback([pool], joined=True) if mode == "async" else contextlib.nullcontext()
                with deferral as tasks:
                    h2d.wait_stream(main)
                    with torch.cuda.stream(h2d):
                        dev_bufs[nb].copy_(pinned[(i + 1) % len(pinned)], non_blocking=True)
                    out = pool.step(*dev_ins[b], groups[i % len(groups)], **kw)
                    d2h.wait_stream(main)
                    with torch.cuda.stream(d2h):
                        host_outs[b].copy_(out, non_blocking=True)
                main.wait_stream(h2d)
                main.wait_stream(d2h)
            return WritebackGraph(graph, tasks, joined=True) if mode == "async" else graph

        e2e_graphs = [e2e_graph(i) for i in range(e2e_period)]
        dev_bufs[0].copy_(pinned[0])  # the first step's inputs; every later step's come with the step before
        for i in range(warmup):
            e2e_graphs[i % e2e_period].replay()
        pool.wait()
        dev_bufs[0].copy_(pinned[0])
        torch.cuda.synchronize()
        barrier()
        e0, e1 = _events()
        e0.record()
        for i in range(steps):
            e2e_graphs[i % e2e_period].replay()
        pool.wait()
        e1.record()
        barrier()
        host_out = host_outs[0]
        res.update(e2e_ms=e0.elapsed_time(e1), h2d=sum(sizes), d2h=host_out.numel() * host_out.element_size())
    return res


def measure_prefill(args, batch, tokens, heads_total, qk_total, steps, warmup, world, rank, device, barrier,
                    e2e=True, clocks=None, seed=3, kda=False):
    """Prefill of ``batch`` prompts of ``tokens`` tokens to their first packed
    states: GDN chunked (config 3), or with ``kda`` the KDA recurrent pass
    (per-key-channel decay) on a {2,4,6} KDA plan of the same shape."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    from stepquant_b200 import synthetic as S
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.quantization import QuantizationPlan

    dim = args.dim
    heads_l, qk_l = heads_total // world, qk_total // world
    gen = torch.Generator(device=device).manual_seed(seed * 1000 + rank)
    cpu_gen = torch.Generator().manual_seed(seed)
    if kda:
        bits = S.kda_widths(heads_total, dim, cpu_gen, choices=(2, 4, 6))[rank * heads_l:(rank + 1) * heads_l]
        plan = QuantizationPlan("kda", bits.to(device), (torch.rand(heads_l, dim, generator=cpu_gen) + 0.5).to(device))
    else:
        widths = S.gdn_widths(heads_total, cpu_gen)[rank * heads_l:(rank + 1) * heads_l]
        plan = QuantizationPlan("gdn", widths[:, None].expand(heads_l, dim).clone().to(device),
                                (torch.rand(heads_l, dim, generator=cpu_gen) + 0.5).to(device))
    pool = PackedStatePool(plan, batch + 1, dim)
    slots = torch.arange(1, batch + 1, device=device)
    total = batch * tokens
    q = torch.randn(1, total, qk_l, dim, device=device, generator=gen).bfloat16()
    k = torch.randn(1, total, qk_l, dim, device=device, generator=gen).bfloat16()
    v = torch.randn(1, total, heads_l, dim, device=device, generator=gen).bfloat16()
    a_log, _ = S.gate_parameters(heads_l, dim, False, gen, device)
    g_shape = (1, total, heads_l, dim) if kda else (1, total, heads_l)
    g = -(a_log.exp()[:, None] if kda else a_log.exp()) * torch.nn.functional.softplus(
        torch.randn(*g_shape, device=device, generator=gen))
    beta = torch.randn(1, total, heads_l, device=device, generator=gen).sigmoid()
    cu = torch.arange(0, total + 1, tokens, device=device, dtype=torch.int32)

    def one_step():
        pool.clear(slots)  # new prompts start from the zero state
        return pool.extend(q, k, v, g, beta, slots, cu)

    for _ in range(warmup):
        one_step()
    barrier()
    start, end = _events()
    barrier()
    if clocks:
        clocks.start()
    start.record()
    for _ in range(steps):
        one_step()
    end.record()
    barrier()
    if clocks:
        clocks.stop()
    res = {"elapsed_ms": start.elapsed_time(end)}
    # per-kernel device times of one step
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        one_step()
        torch.cuda.synchronize()
    kernels, launches = {}, 0
    for ev in prof.key_averages():
        name = ev.key
        if "sq::" in name and ev.device_time_total > 0:
            launches += ev.count
        for short in ("prep_kernel", "state_kernel", "offsets_kernel", "kda_prefill_kernel", "tile_kernel",
                      "fast_kernel", "kda_kernel"):
            if short in name:
                kernels[short] = kernels.get(short, 0.0) + ev.device_time_total / 1e3
    res["kernel_ms"] = kernels
    res["sq_launches"] = launches
    chunk_heads = batch * ((tokens + 63) // 64) * heads_l
    c, kk, vv = 64, dim, dim
    if kda:  # per token and head: the decay product, two column sums and the rank-1 update (7 K V flops)
        res["flops"] = total * heads_l * 7 * kk * vv
    else:
        res["flops"] = chunk_heads * 2 * (3 * c * c * kk + 2 * c * kk * vv + c * kk * vv + c * c * vv)
    # Bytes the path must move: bf16 q, k, v in, fp32 g and beta in, bf16 outputs, the packed first states.
    g_bytes = heads_l * (dim if kda else 1) * 4
    res["bytes"] = total * ((2 * qk_l * dim + 2 * heads_l * dim) * 2 + g_bytes + heads_l * 4) + batch * pool.page_bytes

    if e2e:
        pin = [x.cpu().pin_memory() for x in (q, k, v, g, beta)]
        host_out = torch.empty(v.shape, dtype=torch.bfloat16).pin_memory()

        def e2e_step():
            dev = [x.to(device, non_blocking=True) for x in pin]
            pool.clear(slots)
            out = pool.extend(*dev, slots, cu)
            host_out.copy_(out, non_blocking=True)

        e2e_step()
        barrier()
        e0, e1 = _events()
        e0.record()
        for _ in range(max(1, steps // 4)):
            e2e_step()
        e1.record()
        barrier()
        res.update(e2e_ms=e0.elapsed_time(e1) / max(1, steps // 4) * steps,
                   h2d=sum(x.numel() * x.element_size() for x in pin), d2h=host_out.numel() * host_out.element_size())
    return res


def gather_heads(out, world, group=None):
    """All-gather of per-rank readouts [T, H_local * V] into [T, H * V] in the
    global head order (rank r owns heads [r * H_local, (r + 1) * H_local))."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return out
    parts = torch.empty(world * out.shape[0], out.shape[1], device=out.device, dtype=out.dtype)
    dist.all_gather_into_tensor(parts, out.contiguous(), group=group)  # rank-major concatenation
    return parts.view(world, *out.shape).permute(1, 0, 2).reshape(out.shape[0], world * out.shape[1])


def _rms_norm(x):
    import torch
    # torch's fused kernel (fp32 accumulation, bf16 out): one launch per layer
    # instead of the cast / square / mean / rsqrt / scale / cast chain.
    return torch.nn.functional.rms_norm(x, (x.shape[-1],), eps=1e-6)


def measure_stack(args, batch, heads_total, qk_total, steps, warmup, world, rank, device, barrier, clocks=None,
                  seed=4):
    """Config 4: a stack of GDN layers decoding one token per request per step.

    Value heads (and their qk heads) are tensor-parallel over the ranks.  Per
    layer: RMS-normalised residual -> this rank's column slice of a random-init
    bf16 projection to q, k, v, a, b (cuBLAS) -> ``PackedStatePool.step`` (the
    readout kernel on the compute stream, requantization and repack on the
    writeback stream, joined into the graph) -> NCCL all-gather of the
    readouts [B, H_local * V] -> the gathered readout through a replicated
    random-init output projection, added to the residual.  The prompt goes
    through ``PackedStatePool.extend`` (chunked prefill) first; the decode step
    of all layers is captured once in a CUDA graph (``defer_writeback`` +
    ``WritebackGraph``, joined) and replayed per token.
    """
    import torch
    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile
    from stepquant_b200 import synthetic as S
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.kernels.profiles import stepquant6_profile
    from stepquant_b200.kernels.resources import writeback_resources
    from stepquant_b200.kernels.writeback import WritebackGraph, defer_writeback
    from stepquant_b200.quantization import QuantizationPlan

    dim, hidden, layers, prompt = args.dim, args.hidden, args.layers, args.prompt
    H, HK = heads_total // world, qk_total // world
    o_k, o_v, o_a = HK * dim, 2 * HK * dim, 2 * HK * dim + H * dim
    width = o_a + 2 * H
    gen = torch.Generator(device=device)
    wb_profile = stepquant6_profile("gdn", min(batch, 512))
    resources = writeback_resources(device, wb_profile.sms if args.writeback_sms < 0 else args.writeback_sms)
    wb_stream = resources.stream
    slots = torch.arange(1, batch + 1, device=device)
    # The profile's chunk is per batch tier; with the heads split over ranks one
    # launch of that many requests would leave most SMs idle, so it grows with
    # the rank count (same items per launch as on one GPU).
    chunk = args.writeback_chunk or min(batch, wb_profile.chunk * world)
    stack = []
    page_bytes = 0
    for layer in range(layers):
        cpu_gen = torch.Generator().manual_seed(seed * 1000 + layer)
        widths = S.gdn_widths(heads_total, cpu_gen)[rank * H:(rank + 1) * H]
        plan = QuantizationPlan("gdn", widths[:, None].expand(H, dim).clone().to(device),
                                (torch.rand(heads_total, dim, generator=cpu_gen)[rank * H:(rank + 1) * H] + 0.5).to(device))
        pool = PackedStatePool(plan, batch + 1, dim, writeback_stream=wb_stream, writeback_chunk=chunk)
        page_bytes += pool.page_bytes
        gen.manual_seed((seed * 1000 + layer) * 64 + rank)  # this rank's column slice
        w_in = (torch.randn(hidden, width, device=device, generator=gen) * hidden ** -0.5).bfloat16()
        a_log, dt_bias = S.gate_parameters(H, dim, False, gen, device)
        gen.manual_seed(seed * 1000 + layer + 500_000)  # replicated: identical on every rank
        w_out = (torch.randn(heads_total * dim, hidden, device=device, generator=gen) * (heads_total * dim) ** -0.5).bfloat16()
        stack.append((pool, w_in, w_out, a_log, dt_bias))

    def gather(out):
        return gather_heads(out, world)

    # ---- prompt: chunked prefill of every layer (setup, untimed) ----------------
    tokens = batch * prompt
    gen.manual_seed(seed * 7919)
    h = torch.randn(tokens, hidden, device=device, generator=gen).bfloat16()
    cu = torch.arange(0, tokens + 1, prompt, device=device, dtype=torch.int32)
    for pool, w_in, w_out, a_log, dt_bias in stack:
        proj = _rms_norm(h) @ w_in
        q = proj[:, :o_k].view(1, tokens, HK, dim)
        k = proj[:, o_k:o_v].view(1, tokens, HK, dim)
        v = proj[:, o_v:o_a].view(1, tokens, H, dim)
        a, b = proj[:, o_a:o_a + H].float(), proj[:, o_a + H:].float()
        g = (-a_log.exp() * torch.nn.functional.softplus(a + dt_bias))[None]
        out = pool.extend(q, k, v, g, b.sigmoid()[None], slots, cu, scale=dim ** -0.5)
        h = torch.addmm(h, gather(out.reshape(tokens, H * dim)), w_out)
        del proj, q, k, v, a, b, g, out
    prompt_state = float(h.float().square().mean().sqrt())
    del h
    torch.cuda.synchronize()

    # ---- decode: one token per request per step, all layers in one graph --------
    embeds = 4
    gen.manual_seed(seed * 7919 + 1)
    inputs = torch.randn(embeds, batch, hidden, device=device, generator=gen).bfloat16()
    x_in = torch.empty(batch, hidden, device=device, dtype=torch.bfloat16)
    result = torch.empty(batch, device=device, dtype=torch.float32)
    pools = [layer[0] for layer in stack]

    def decode_step():
        h = x_in
        for pool, w_in, w_out, a_log, dt_bias in stack:
            proj = _rms_norm(h) @ w_in
            out = pool.step(proj[:, :o_k], proj[:, o_k:o_v], proj[:, o_v:o_a], proj[:, o_a:o_a + H].float(),
                            proj[:, o_a + H:].float(), slots, normalize=True, scale=dim ** -0.5, a_log=a_log,
                            dt_bias=dt_bias)
            h = torch.addmm(h, gather(out.reshape(batch, H * dim)), w_out)  # residual add in the GEMM
        result.copy_(h.float().sum(-1))

    x_in.copy_(inputs[0])
    decode_step()  # eager: cuBLAS handles, NCCL communicator, pool workspaces
    for pool in pools:
        pool.wait()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        with defer_writeback(pools, joined=True) as tasks:
            decode_step()
    replay = WritebackGraph(graph, tasks, joined=True)

    def one_step(i):
        x_in.copy_(inputs[i % embeds])
        replay.replay()

    for i in range(warmup):
        one_step(i)
    barrier()
    start, end = _events()
    barrier()
    if clocks:
        clocks.start()
    start.record()
    for i in range(steps):
        one_step(i)
    for pool in pools:
        pool.wait()
    end.record()
    barrier()
    if clocks:
        clocks.stop()
    res = {"elapsed_ms": start.elapsed_time(end), "page_bytes": page_bytes, "prompt_rms": prompt_state, "chunk": chunk,
           "writeback_sms": resources.actual_sms,
           "finite": bool(torch.isfinite(result).all())}

    # Device time of one replay by kernel family (ranks aligned first, so the
    # all-gather does not absorb another rank's start-up skew).
    barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        one_step(0)
        for pool in pools:
            pool.wait()
        torch.cuda.synchronize()
    fam = {"state_readout": 0.0, "state_writeback": 0.0, "gemm": 0.0, "nccl": 0.0, "other": 0.0}
    launches = 0
    for ev in prof.key_averages():
        name, ms = ev.key, ev.device_time_total / 1e3
        if ms <= 0:
            continue
        if "fast_kernel<3," in name or "fast_kernel<(int)3," in name:
            fam["state_readout"] += ms
            launches += ev.count
        elif "fast_kernel<4," in name or "fast_kernel<(int)4," in name or "tile_kernel" in name:
            fam["state_writeback"] += ms
            launches += ev.count
        elif "sq::" in name:
            fam["other"] += ms
            launches += ev.count
        elif "nccl" in name.lower():
            fam["nccl"] += ms
        elif "gemm" in name.lower() or "nvjet" in name.lower() or "cutlass" in name.lower():
            fam["gemm"] += ms
        else:
            fam["other"] += ms
    res["kernel_ms"] = fam
    res["sq_launches"] = launches

    # End to end: each step's embeddings from pinned host memory, the step's
    # per-request result back to the host.
    pin = inputs.cpu().pin_memory()
    host_res = torch.empty(batch, dtype=torch.float32).pin_memory()

    def e2e_step(i):
        x_in.copy_(pin[i % embeds], non_blocking=True)
        replay.replay()
        host_res.copy_(result, non_blocking=True)

    e2e_step(0)
    barrier()
    e0, e1 = _events()
    e0.record()
    for i in range(steps):
        e2e_step(i)
    for pool in pools:
        pool.wait()
    e1.record()
    barrier()
    res.update(e2e_ms=e0.elapsed_time(e1), h2d=batch * hidden * 2, d2h=batch * 4)
    for pool in pools:
        pool.wait()
    torch.cuda.synchronize()
    # Graphs holding NCCL work are released before the process group goes.
    del replay, graph, tasks
    return res


def main():
    args = parse_args()
    # Library and NCCL messages written to fd 1 go to stderr; the result line
    # alone goes to the original stdout.
    result_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    sys.stdout = sys.stderr
    global _result_out
    _result_out = result_out
    if args.impl == "reference":
        reference_arm(args)
        return
    if args.impl == "reference-gpu":
        reference_gpu_arm(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} does not match WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(*values):
        t = torch.tensor(values, device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def sum_over_ranks(*values):
        t = torch.tensor(values, device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t)
        return t.tolist()

    workload = args.workload
    kda = workload == "kda-decode"
    batch = args.batch if args.batch else (512 if kda or workload == "gdn-stack" else
                                           32 if workload in ("gdn-prefill", "kda-prefill") else 256)
    heads = args.heads
    qk_heads = args.qk_heads if args.qk_heads else (heads if kda or workload == "kda-prefill" else heads // 2)
    if heads % world or qk_heads % world:
        raise SystemExit("heads must divide evenly over ranks")
    clocks = ClockSampler(local)
    peak_hbm, peak_hbm_kind = measured_peak()
    line = {"metric": METRIC, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic"}

    if workload == "gdn-stack":
        res = measure_stack(args, batch, heads, qk_heads, args.steps, args.warmup, world, rank, device, barrier,
                            clocks=clocks)
        elapsed_ms, e2e_ms = max_over_ranks(res["elapsed_ms"], res["e2e_ms"])
        fam = res["kernel_ms"]
        state_ms = fam["state_readout"] + fam["state_writeback"]
        ms_per_step = elapsed_ms / args.steps
        units = batch * args.steps
        page_io, other_io = algorithmic_bytes(res["page_bytes"], heads // world, qk_heads // world, batch, args.dim)
        other_io *= args.layers
        achieved = (page_io + other_io) / (state_ms / 1e3) / 1e9 if state_ms else None
        line.update({
            "metric": "stack decode tokens/s", "unit": "tokens/s", "value": units / (elapsed_ms / 1e3),
            "ms_per_step": ms_per_step,
            "config": {"workload": "gdn-stack-l%d-b%d-h%d-hidden%d (config 4)" % (args.layers, batch, heads, args.hidden),
                       "layers": args.layers, "batch": batch, "hidden": args.hidden, "heads": heads,
                       "qk_heads": qk_heads, "dim": args.dim, "prompt_tokens": args.prompt,
                       "decode_tokens_timed": args.steps, "plan": "stepquant6 synthetic per layer",
                       "parallelism": f"tp{world} (value heads), NCCL all-gather of each layer's readout",
                       "graph": "one CUDA graph per decode token (all layers), writeback joined",
                       "writeback_chunk": res["chunk"], "writeback_sms": res["writeback_sms"],
                       "weights": "random-init bf16 in/out projections",
                       "l2": "pages of %d layers (%.0f MB per GPU) > L2" % (args.layers, (batch + 1) * res["page_bytes"] / 1e6)},
            "kernel_ms_per_step": fam,
            "state_update_share": state_ms / max(sum(fam.values()), 1e-9),
            "state_update_share_basis": "summed device time of the token's kernels (streams overlap)",
            "roofline": {"kernel": "state kernels (readout + writeback, all layers)", "bound": "hbm",
                         "achieved": achieved, "peak": peak_hbm, "unit": "GB/s",
                         "frac": achieved / peak_hbm if achieved else None, "traffic": None,
                         "peak_source": peak_hbm_kind, "algorithmic_bytes_per_step": page_io + other_io},
            "e2e": {"value": units / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": res["h2d"],
                    "d2h_bytes_per_step": res["d2h"]},
            "gpu_launches": res["sq_launches"] * args.steps,
            "finite": res["finite"],
        })
    elif workload == "gdn-prefill":
        res = measure_prefill(args, batch, args.tokens, heads, qk_heads, args.steps, args.warmup, world, rank, device,
                              barrier, e2e=True, clocks=clocks)
        elapsed_ms, e2e_ms = max_over_ranks(res["elapsed_ms"], res["e2e_ms"])
        flops, nbytes = sum_over_ranks(res["flops"], res["bytes"])
        units = batch * args.tokens * args.steps
        peak_tf, peak_tf_kind = measured_peak("bf16_tflops")
        peak_hbm, peak_hbm_kind = measured_peak("hbm_gbs")
        kern = res["kernel_ms"]
        dom_ms = sum(kern.values())
        achieved_tf = flops / world / (dom_ms / 1e3) / 1e12 if dom_ms else None
        achieved_gbs = nbytes / world / (dom_ms / 1e3) / 1e9 if dom_ms else None
        # DRAM bytes of prep_kernel + state_kernel per launch from ncu on 4 prompts (259.0 + 296.8 MB), scaled by
        # the prompts processed: traffic grows in proportion (one record per chunk and head).
        traffic = 555.8e6 * batch / 4 if (args.tokens, heads // world, qk_heads // world) == (2048, 32, 16) else None
        # The prefill is reported against the tensor roofline; the HBM view sits beside it, with the resource
        # that takes longer at its peak (at config 3 the bytes, 0.25 ms, over the flops, 0.21 ms).
        hbm = {"achieved": achieved_gbs, "peak": peak_hbm, "unit": "GB/s",
               "frac": achieved_gbs / peak_hbm if achieved_gbs else None, "traffic": traffic,
               "peak_source": peak_hbm_kind, "algorithmic_bytes_per_launch": nbytes / world}
        slower = "hbm" if nbytes / (peak_hbm * 1e9) >= flops / (peak_tf * 1e12) else "tensor"
        line.update({
            "metric": "chunked-prefill tokens/s", "unit": "tokens/s", "value": units / (elapsed_ms / 1e3),
            "ms_per_step": elapsed_ms / args.steps, "dtype": "bf16",
            "config": {"workload": "gdn-prefill-b%d-t%d-h%d-k128 (config 3)" % (batch, args.tokens, heads),
                       "batch": batch, "tokens": args.tokens, "chunk": 64, "heads": heads, "qk_heads": qk_heads,
                       "plan": "stepquant6 synthetic (first packed state)", "parallelism": f"tp{world} (value heads)",
                       "l2": "inputs > L2 (%.0f MB of q/k/v per GPU)" % ((2 * qk_heads + heads) // world * 128 * 2 * batch * args.tokens / 1e6)},
            "kernel_ms": kern,
            "roofline": {"kernel": "prep_kernel + state_kernel + offsets_kernel + fast_kernel (one prefill call)",
                         "bound": "tensor", "achieved": achieved_tf, "peak": peak_tf, "unit": "TFLOP/s",
                         "frac": achieved_tf / peak_tf if achieved_tf else None, "traffic": traffic,
                         "traffic_unit": "bytes", "peak_source": peak_tf_kind,
                         "algorithmic_flops_per_launch": flops / world, "hbm": hbm,
                         "slower_at_peak": slower},
            "e2e": {"value": units / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": res["h2d"],
                    "d2h_bytes_per_step": res["d2h"]},
            "gpu_launches": args.steps * 5,
        })
    elif workload == "kda-prefill":
        res = measure_prefill(args, batch, args.tokens, heads, qk_heads, args.steps, args.warmup, world, rank, device,
                              barrier, e2e=True, clocks=clocks, kda=True)
        elapsed_ms, e2e_ms = max_over_ranks(res["elapsed_ms"], res["e2e_ms"])
        (flops,) = sum_over_ranks(res["flops"])
        units = batch * args.tokens * args.steps
        kern = res["kernel_ms"]
        kp = kern.get("kda_prefill_kernel", 0.0)
        # The recurrent pass runs on the FP32 pipe (packed FMUL2 / FFMA2); its
        # roofline is the nominal fp32 rate, 148 SMs x 128 lanes x 2 flops x 1.965 GHz.
        peak = 148 * 128 * 2 * 1.965e9 / 1e12
        achieved = flops / world / (kp / 1e3) / 1e12 if kp else None
        line.update({
            "metric": "prefill tokens/s", "unit": "tokens/s", "value": units / (elapsed_ms / 1e3),
            "ms_per_step": elapsed_ms / args.steps, "dtype": "f32",
            "config": {"workload": "kda-prefill-b%d-t%d-h%d-k128" % (batch, args.tokens, heads),
                       "batch": batch, "tokens": args.tokens, "heads": heads, "qk_heads": qk_heads,
                       "plan": "{2,4,6} KDA rows, 2% fp16 pivot rows (first packed state)",
                       "parallelism": f"tp{world} (value heads)", "l2": "inputs > L2"},
            "kernel_ms": kern,
            "roofline": {"kernel": "kda_prefill_kernel", "bound": "fp32", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak if achieved else None, "traffic": None,
                         "peak_source": "nominal fp32 FMA rate (no measured figure for the FP32 pipe)",
                         "algorithmic_flops_per_launch": flops / world},
            "e2e": {"value": units / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": res["h2d"],
                    "d2h_bytes_per_step": res["d2h"]},
            "gpu_launches": res["sq_launches"] * args.steps,
        })
    else:
        res = measure_decode(args, kda, batch, heads, qk_heads, args.steps, args.warmup, world, rank, device, barrier,
                             mode=args.mode, e2e=True, clocks=clocks, warm_steps=args.warm_steps,
                             slot_groups=args.slot_groups, seed=2 if kda else args.seed,
                             kda_widths=tuple(int(w) for w in args.kda_widths.split(",")))
        elapsed_ms, e2e_ms = max_over_ranks(res["elapsed_ms"], res["e2e_ms"])
        page_io, other_io = res["algorithmic"]
        job_page_bytes, step_bytes = (int(x) for x in sum_over_ranks(res["page_bytes"], page_io + other_io))
        units = batch * heads * args.steps
        kernel_ms = res["kernel_ms"]
        if args.mode == "sync":
            dominant, dom_bytes, dom_ms = "sq_step (fused)", page_io + other_io, kernel_ms.get("step")
        else:
            rd, wb = kernel_ms.get("readout", 0.0), kernel_ms.get("writeback", 0.0)
            if wb >= rd:
                dominant, dom_bytes, dom_ms = "sq_writeback", page_io, wb
            else:
                dominant, dom_bytes, dom_ms = "sq_readout", page_io // 2 + other_io, rd
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9 if dom_ms else None
        # DRAM read + write bytes of one launch at this workload, from an ncu capture made
        # outside the bench (ncu cannot run inside a timed region); None for other shapes.
        ncu_traffic = {"sq_step (fused)": 153.8e6, "sq_writeback": 157.9e6, "sq_readout": 113.5e6}
        default_shape = (not kda, batch, heads, qk_heads, args.dim, world, args.pivot_heads, args.two_bit_heads) == \
            (True, 256, 32, 16, 128, 1, 1, 0)
        name = ("kda-decode-b%d-h%d-k128 (config 2)" if kda else "gdn-decode-b%d-h%d-k128 (config 1)") % (batch, heads)
        kw_desc = "{%s}" % args.kda_widths
        plan_desc = (("stepquant4 reference-legal twin: " if args.kda_widths == "2,4,6" else
                      "config 2's plan (3/5-bit width extension): ") + "row widths %s at 30/50/20, 2%% fp16 pivot rows"
                     % kw_desc if kda else
                     "stepquant6 synthetic, widths {4,6,8} 25/50/25, pivot heads %d" % args.pivot_heads +
                     (", 2-bit heads %d" % args.two_bit_heads if args.two_bit_heads else ""))
        line.update({
            "value": units / (elapsed_ms / 1e3), "ms_per_step": elapsed_ms / args.steps,
            "config": {"workload": name, "batch": batch, "heads": heads, "qk_heads": qk_heads, "dim": args.dim,
                       "mode": args.mode, "writeback": args.mode == "async", "plan": plan_desc,
                       "page_bytes_per_request": job_page_bytes, "l2": "inputs > L2: slots rotate over %d groups "
                       "(%.0f MB of pages per GPU)" % (args.slot_groups, (args.slot_groups * batch + 1) * res["page_bytes"] / 1e6),
                       "parallelism": f"tp{world} (value heads)"},
            "request_steps_per_s": units / heads / (elapsed_ms / 1e3),
            "algorithmic_gb_per_s": step_bytes * args.steps / (elapsed_ms / 1e3) / 1e9,
            "hbm_fraction_whole_step": step_bytes / world * args.steps / (elapsed_ms / 1e3) / 1e9 / peak_hbm,
            "kernel_ms": kernel_ms,
            "roofline": {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": peak_hbm, "unit": "GB/s",
                         "frac": achieved / peak_hbm if achieved else None,
                         "traffic": ncu_traffic.get(dominant) if default_shape else None, "peak_source": peak_hbm_kind,
                         "algorithmic_bytes_per_launch": dom_bytes},
            "e2e": {"value": units / (e2e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": res["h2d"],
                    "d2h_bytes_per_step": res["d2h"]},
            # readout (or fused step), writeback; the pivot-head readout; the 2-bit heads' readout and writeback
            "gpu_launches": args.steps * ((2 if args.mode == "async" else 1) + (1 if res["pivot_heads_local"] else 0) +
                                          ((2 if args.mode == "async" else 1) if res["two_bit_heads_local"] else 0)),
        })
    line["clocks"] = clocks.summary()

    # Short measurements of the other configurations (default workload only), on
    # the same ranks: value heads sharded as in config 1, times max over ranks.
    if workload == "gdn-decode" and not args.no_secondary:
        sec = {}
        for widths, key, note in (
                ((2, 4, 6), "kda-decode-b512-h32-k128 (config 2)",
                 "reference-legal twin plan: row widths {2,4,6} at 30/50/20, 2% fp16 pivot rows; "
                 "64 warm-up steps, 2 slot groups"),
                ((3, 4, 6), "kda-decode-b512-h32-k128-w346 (config 2, width extension)",
                 "config 2's own plan: row widths {3,4,6} at 30/50/20, 2% fp16 pivot rows (3-bit rows are this "
                 "build's extension; the reference rejects them)")):
            r2 = measure_decode(args, True, 512, 32, 32, 5, 3, world, rank, device, barrier, mode="async", e2e=False,
                                warm_steps=64, slot_groups=2, seed=2, kda_widths=widths)
            (ms2,) = max_over_ranks(r2["elapsed_ms"])
            (pb2,) = sum_over_ranks(r2["page_bytes"])
            sec[key] = {"value": 512 * 32 * 5 / (ms2 / 1e3), "unit": UNIT, "ms_per_step": ms2 / 5,
                        "kernel_ms": r2["kernel_ms"], "steps": 5, "mode": "async",
                        "page_bytes_per_request": int(pb2), "note": note}
        r3 = measure_prefill(args, 32, 2048, 32, 16, 5, 2, world, rank, device, barrier, e2e=False)
        (ms3,) = max_over_ranks(r3["elapsed_ms"])
        flops3, bytes3 = sum_over_ranks(r3["flops"], r3["bytes"])
        peak_tf, peak_tf_kind = measured_peak("bf16_tflops")
        peak_hbm, _ = measured_peak("hbm_gbs")
        pk = sum(r3["kernel_ms"].values())
        sec["gdn-prefill-b32-t2048-h32-k128 (config 3)"] = {
            "value": 32 * 2048 * 5 / (ms3 / 1e3), "unit": "tokens/s", "ms_per_step": ms3 / 5,
            "kernel_ms": r3["kernel_ms"], "steps": 5,
            "hbm_frac": (bytes3 / world / (pk / 1e3) / 1e9 / peak_hbm) if pk else None,
            "tensor_tflops": flops3 / world / (pk / 1e3) / 1e12 if pk else None,
            "tensor_frac": (flops3 / world / (pk / 1e3) / 1e12 / peak_tf) if pk else None,
            "peak_source": peak_tf_kind}
        r5 = measure_prefill(args, 32, 2048, 32, 32, 3, 1, world, rank, device, barrier, e2e=False, kda=True)
        (ms5,) = max_over_ranks(r5["elapsed_ms"])
        (flops5,) = sum_over_ranks(r5["flops"])
        pk5 = sum(r5["kernel_ms"].values())
        # fp32 FMA pipe, nominal: 148 SMs x 128 lanes x 2 flops x 1.965 GHz
        fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        kp5 = r5["kernel_ms"].get("kda_prefill_kernel", 0.0)
        sec["kda-prefill-b32-t2048-h32-k128"] = {
            "value": 32 * 2048 * 3 / (ms5 / 1e3), "unit": "tokens/s", "ms_per_step": ms5 / 3,
            "kernel_ms": r5["kernel_ms"], "steps": 3,
            "fp32_tflops": flops5 / world / (kp5 / 1e3) / 1e12 if kp5 else None,
            "fp32_frac_of_nominal": flops5 / world / (kp5 / 1e3) / 1e12 / fp32_peak if kp5 else None,
            "note": "KDA prefill to the first packed states ({2,4,6} KDA plan, H = HK = 32): decode, the recurrent "
                    "fp32 state pass (kda_prefill_kernel, 7 K V flops per token and head), encode"}
        r4 = measure_stack(args, 512, 32, 16, 5, 2, world, rank, device, barrier)
        ms4_all, e2e4 = max_over_ranks(r4["elapsed_ms"], r4["e2e_ms"])
        fam, ms4 = r4["kernel_ms"], ms4_all / 5
        sec["gdn-stack-l%d-b512-h32-hidden%d (config 4)" % (args.layers, args.hidden)] = {
            "value": 512 * 5 / (ms4_all / 1e3), "unit": "tokens/s", "ms_per_step": ms4,
            "e2e": 512 * 5 / (e2e4 / 1e3), "kernel_ms_per_step": fam,
            # The writeback of layer l runs beside layer l+1 on its own stream, so kernel times
            # summed over a token exceed the token's wall time: the share is of the summed time.
            "state_update_share": (fam["state_readout"] + fam["state_writeback"]) / max(sum(fam.values()), 1e-9),
            "state_update_share_basis": "summed device time of the token's kernels (streams overlap)", "steps": 5,
            "finite": r4["finite"],
            "note": "%d GDN layers, prompt %d tokens then decode; one CUDA graph per decode token (writeback joined), "
                    "%s" % (args.layers, args.prompt,
                            "1 GPU (the all-gather is the identity)" if world == 1 else
                            "tp%d: NCCL all-gather of each layer's readout inside the graph" % world)}
        line["secondary"] = sec

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if not args.no_cpu_baseline and world == 1 and workload == "gdn-decode":
        cpu = cpu_reference(args, heads, qk_heads, batch, 100, 1, args.cpu_seconds)
    line["cpu_baseline"] = cpu
    emit(line)


if __name__ == "__main__":
    main()
