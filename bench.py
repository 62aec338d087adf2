#!/usr/bin/env python
"""Packed-state GDN decode benchmark on 1..8 B200s.

One *step* is one decode step of one GDN layer over the whole batch: for every
(request, value head) the packed state page is unpacked, the gated delta rule
applied, o = S^T q read out, the state requantized (fit_state), repacked and
written back.  Asynchronous writeback is on (config 1): the readout kernel runs
on the compute stream and the requantization on a writeback stream, and a
step is complete when both are.  ``--mode sync`` times the fused single-kernel
step instead.

Workload: Qwen-Next-style layer, 16 qk heads / 32 value heads, K = V = 128,
batch 256, stepquant6 synthetic plan (seed 1: per-head widths {4, 6, 8} at
25/50/25, impact factors from a 256-step fp32 warm-up).  Value heads (and their
qk heads) are sharded over ranks as tensor parallelism does; no collective runs
in the timed state path.  Requests rotate over 4 groups of slots (a 420 MB pool
per GPU at N = 1, larger than the 126 MB L2), so each step reads pages that are
not L2-resident.

Prints one JSON line on rank 0.  ``--impl reference`` times the reference's CPU
path (StateCodec.decode -> delta_step -> StateCodec.encode, restated in numpy
by the oracle) on the host cores instead.
"""
import argparse
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
    p.add_argument("--impl", choices=("stepquant_b200", "reference"), default="stepquant_b200")
    p.add_argument("--mode", choices=("async", "sync"), default="async")
    p.add_argument("--batch", type=int, default=256)
    p.add_argument("--heads", type=int, default=32)
    p.add_argument("--qk-heads", type=int, default=16)
    p.add_argument("--dim", type=int, default=128)
    p.add_argument("--pivot-heads", type=int, default=0)
    p.add_argument("--slot-groups", type=int, default=4)
    p.add_argument("--warm-steps", type=int, default=256)
    p.add_argument("--seed", type=int, default=1)
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
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


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def algorithmic_bytes(pool_page_bytes, heads_local, qk_local, batch, dim):
    """Bytes one decode step must move (per rank): pages read+written, bf16 q/k/v in, gates, bf16 out."""
    pages = 2 * pool_page_bytes * batch
    inputs = batch * (2 * qk_local * dim + heads_local * dim) * 2
    gates = batch * heads_local * 8
    output = batch * heads_local * dim * 2
    return pages, inputs + gates + output


# ---------------------------------------------------------------------------
# CPU reference arm / baseline (oracle port of the reference's torch path)
# ---------------------------------------------------------------------------

_cpu_state = {}


def _cpu_init(seed, heads, qk_heads, dim, requests):
    import numpy as np
    from oracle import stepquant_oracle as O
    rng = np.random.default_rng(seed)
    widths = np.array(([4] * (heads // 4) + [6] * (heads - 2 * (heads // 4)) + [8] * (heads // 4)))
    rng.shuffle(widths)
    bits = np.repeat(widths[:, None], dim, 1)
    plan = O.Plan("gdn", bits, (rng.random((heads, dim)) + 0.5).astype(np.float32))
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
    plan = s["plan"]
    state = O.codec_decode(s["packed"], plan)
    qp, kp, g, beta = O.prepare_inputs(q, k, a, b, plan.bits.shape[0], kda=False, normalize=True,
                                       scale=s["dim"] ** -0.5, a_log=a_log, dt_bias=dt_bias)
    _, updated = O.delta_step(state, qp, kp, v, g, beta)
    s["packed"] = O.codec_encode(updated, plan)
    return int(q.shape[0])


def cpu_reference(args, heads, qk_heads, steps, warmup, budget_seconds):
    """Time the CPU port with one spawned worker per host core; returns a dict."""
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    requests = 1
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores, initializer=_cpu_init, initargs=(args.seed, heads, qk_heads, args.dim, requests)) as pool:
        for _ in range(max(1, warmup)):
            pool.map(_cpu_step, range(cores))
        times = []
        t_end = time.perf_counter() + budget_seconds
        for _ in range(steps):
            t0 = time.perf_counter()
            done = sum(pool.map(_cpu_step, range(cores)))
            times.append(time.perf_counter() - t0)
            if time.perf_counter() > t_end:
                break
    per_step = statistics.median(times)
    updates = done * heads / per_step
    return {"value": updates, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{cores} workers x {requests} request x {heads} heads (K=V={args.dim}) per step, "
                      f"{len(times)} steps, median step {per_step * 1e3:.1f} ms"}


def reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    res = cpu_reference(args, args.heads, args.qk_heads, args.steps, args.warmup,
                        max(20.0, args.cpu_seconds * 3))
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            # one full batch-step at the sampled rate
            "ms_per_step": args.batch * args.heads / res["value"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "gdn-decode-b256-h32-k128 (config 1), CPU port of the reference torch path",
                       "batch": args.batch, "heads": args.heads, "qk_heads": args.qk_heads, "dim": args.dim},
            "cpu_baseline": res, "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                                          "d2h_bytes_per_step": 0}}
    emit(line)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

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
    if args.heads % world or args.qk_heads % world:
        raise SystemExit("heads must divide evenly over ranks")

    from stepquant_b200 import _native as N
    from stepquant_b200 import synthetic as S
    from stepquant_b200.kernels.pool import PackedStatePool
    from stepquant_b200.quantization import QuantizationPlan

    heads_l, qk_l, dim, batch = args.heads // world, args.qk_heads // world, args.dim, args.batch
    gen = torch.Generator(device=device).manual_seed(args.seed * 1000 + rank)
    cpu_gen = torch.Generator().manual_seed(args.seed)
    widths = S.gdn_widths(args.heads, cpu_gen, args.pivot_heads)[rank * heads_l:(rank + 1) * heads_l]
    a_log, dt_bias = S.gate_parameters(heads_l, dim, False, gen, device)
    requests = batch * args.slot_groups
    slots_total = requests + 1

    # fp32 warm-up state (the FP32 pool kernel) and row-impact statistics.
    fp32 = torch.zeros(slots_total, heads_l, dim, dim, device=device)
    warm_slots = torch.arange(1, slots_total, device=device)
    out_scratch = torch.empty(requests, heads_l, dim, device=device, dtype=torch.bfloat16)
    omega = torch.zeros(heads_l, dim, device=device, dtype=torch.float64)
    for _ in range(args.warm_steps):
        inp = S.draw_inputs(requests, heads_l, qk_l, dim, dim, False, gen, device)
        st = N.SqStepArgs(inp.q.data_ptr(), inp.k.data_ptr(), inp.v.data_ptr(), inp.q.stride(0), inp.k.stride(0),
                          inp.v.stride(0), qk_l, N.SQ_BF16, inp.a.data_ptr(), inp.b.data_ptr(), N.SQ_F32, 1,
                          a_log.data_ptr(), dt_bias.data_ptr(), dim ** -0.5, 0, out_scratch.data_ptr())
        N.check(N.lib().sq_fp32_step(N.ptr(fp32), slots_total, heads_l, dim, dim, 0, N.ptr(warm_slots), requests,
                                     ctypes.byref(st), None, N.stream_handle()))
        q, k, g, beta = S.prepared(inp, heads_l, dim, False, a_log, dt_bias)
        omega += S.row_impact(q, k, g, beta).double().sum(0)
    impact = S.impact_factors(omega / (args.warm_steps * requests))
    plan = QuantizationPlan("gdn", widths[:, None].expand(heads_l, dim).clone().to(device), impact.to(device))

    stream = torch.cuda.Stream(device) if args.mode == "async" else None
    pool = PackedStatePool(plan, slots_total, dim, writeback_stream=stream)
    pool.encode(fp32[1:], warm_slots)
    del fp32
    groups = [torch.arange(1 + g * batch, 1 + (g + 1) * batch, device=device) for g in range(args.slot_groups)]
    inputs = [S.draw_inputs(batch, heads_l, qk_l, dim, dim, False, gen, device) for _ in range(4)]
    kw = dict(normalize=True, scale=dim ** -0.5, a_log=a_log, dt_bias=dt_bias)

    # Per-kernel CUDA events on the stream each kernel runs on.
    marks = {"readout": [], "writeback": [], "step": []}
    recording = [False]
    finish = pool._finish_update

    def timed_finish(*tensors, **kwargs):
        if recording[0]:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            finish(*tensors, **kwargs)
            e1.record()
            marks["writeback"].append((e0, e1))
        else:
            finish(*tensors, **kwargs)

    pool._finish_update = timed_finish

    def one_step(i):
        inp = inputs[i % len(inputs)]
        pool.wait()
        if recording[0]:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        out = pool.step(inp.q, inp.k, inp.v, inp.a, inp.b, groups[i % len(groups)], **kw)
        if recording[0]:
            e1.record()
            marks["readout" if args.mode == "async" else "step"].append((e0, e1))
        return out

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    clocks = ClockSampler(local)
    for i in range(args.warmup):
        one_step(i)
    pool.wait()
    barrier()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    clocks.start()
    recording[0] = True
    start.record()
    for i in range(args.steps):
        one_step(i)
    pool.wait()
    end.record()
    recording[0] = False
    barrier()
    clocks.stop()
    elapsed_ms = start.elapsed_time(end)
    kernel_ms = {name: sum(a.elapsed_time(b) for a, b in ev) / max(1, len(ev)) for name, ev in marks.items() if ev}
    pool.check_status()

    # End to end through the public API with host buffers.
    # Each step's inputs (q, k, v bf16; a, b fp32) packed in one pinned host
    # buffer and copied with one H2D transfer; the output comes back with one D2H.
    fields = [(x.shape, x.dtype) for x in (inputs[0].q, inputs[0].k, inputs[0].v, inputs[0].a, inputs[0].b)]
    sizes = [math.prod(sh) * torch.tensor([], dtype=dt).element_size() for sh, dt in fields]
    offsets = [0]
    for n in sizes:
        offsets.append(offsets[-1] + (n + 255) // 256 * 256)
    pinned = []
    for x in inputs:
        buf = torch.empty(offsets[-1], dtype=torch.uint8).pin_memory()
        for t, o, n in zip((x.q, x.k, x.v, x.a, x.b), offsets, sizes):
            buf[o:o + n].copy_(t.contiguous().view(-1).view(torch.uint8).cpu())
        pinned.append(buf)
    dev_buf = torch.empty(offsets[-1], dtype=torch.uint8, device=device)
    dev_in = tuple(dev_buf[o:o + n].view(dt).view(sh) for (sh, dt), o, n in zip(fields, offsets, sizes))
    host_out = torch.empty(batch, heads_l, dim, dtype=torch.bfloat16).pin_memory()
    h2d = sum(sizes)
    d2h = host_out.numel() * host_out.element_size()

    def e2e_step(i):
        dev_buf.copy_(pinned[i % len(pinned)], non_blocking=True)
        out = pool.step(*dev_in, groups[i % len(groups)], **kw)
        host_out.copy_(out, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    pool.wait()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        e2e_step(i)
    pool.wait()
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    times = torch.tensor([elapsed_ms, e2e_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms = times.tolist()

    units = args.batch * args.heads * args.steps
    value = units / (elapsed_ms / 1e3)
    e2e_value = units / (e2e_ms / 1e3)

    page_bytes = pool.page_bytes
    page_io, other_io = algorithmic_bytes(page_bytes, heads_l, qk_l, batch, dim)
    # Each rank's plan covers its own value heads: job totals are sums over ranks.
    totals = torch.tensor([page_bytes, page_io + other_io], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(totals)
    job_page_bytes, step_bytes = (int(t) for t in totals.tolist())
    peak, peak_kind = measured_peak()
    if args.mode == "sync":
        dominant, dom_bytes = "sq_step (fused)", page_io + other_io
        dom_ms = kernel_ms.get("step")
    else:
        rd, wb = kernel_ms.get("readout", 0.0), kernel_ms.get("writeback", 0.0)
        if wb >= rd:
            dominant, dom_bytes, dom_ms = "sq_writeback", page_io, wb
        else:
            dominant, dom_bytes, dom_ms = "sq_readout", page_io // 2 + other_io, rd
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9 if dom_ms else None
    # dram read + write bytes per launch from one ncu capture of this workload
    # (profiles/fast_kernel_gdn_b256.md); None for other shapes.
    ncu_traffic = {"sq_step (fused)": 160.6e6, "sq_writeback": 162.3e6, "sq_readout": 116.7e6}
    default_shape = (args.batch, args.heads, args.qk_heads, dim, world) == (256, 32, 16, 128, 1)
    traffic = ncu_traffic.get(dominant) if default_shape else None

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    cpu = None
    if not args.no_cpu_baseline and world == 1:
        cpu = cpu_reference(args, args.heads, args.qk_heads, 100, 1, args.cpu_seconds)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "gdn-decode-b256-h32-k128 (config 1)", "batch": batch, "heads": args.heads,
                   "qk_heads": args.qk_heads, "dim": dim, "mode": args.mode, "writeback": args.mode == "async",
                   "plan": "stepquant6 synthetic, widths {4,6,8} 25/50/25, pivot heads %d" % args.pivot_heads,
                   "page_bytes_per_request": job_page_bytes, "l2": "inputs > L2: slots rotate over %d groups "
                   "(%.0f MB of pages per GPU)" % (args.slot_groups, slots_total * page_bytes / 1e6),
                   "parallelism": f"tp{world} (value heads)"},
        "request_steps_per_s": value / args.heads,
        "algorithmic_gb_per_s": step_bytes * args.steps / (elapsed_ms / 1e3) / 1e9,
        "hbm_fraction_whole_step": step_bytes / world * args.steps / (elapsed_ms / 1e3) / 1e9 / peak,
        "kernel_ms": kernel_ms,
        "roofline": {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if achieved else None, "traffic": traffic, "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": dom_bytes},
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": args.steps * (2 if args.mode == "async" else 1),
        "cpu_baseline": cpu,
    }
    emit(line)


if __name__ == "__main__":
    main()
