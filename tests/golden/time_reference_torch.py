"""Time the reference's own CPU path beside this repository's numpy port of it.

The reference is Python (torch) and cannot travel to the GPU box, so the
benchmark's CPU baseline there is the numpy port (``oracle``).  This script,
run in a container that has the reference checkout, times both on the same
host cores with the config-1 shapes (32 value heads over 16 qk heads,
K = V = 128, widths {4, 6, 8} at 8/16/8), one decode step of ``--requests``
requests: ``StateCodec.decode -> delta_step -> StateCodec.encode`` with the
gate/normalisation prologue, as ``bench.py --impl reference`` runs the port.

    python tests/golden/time_reference_torch.py --reference <checkout> [--requests 16] [--threads 8]

Prints one JSON line: seconds per update for each, and their ratio.
"""
import argparse
import json
import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--reference", required=True)
    p.add_argument("--requests", type=int, default=16)
    p.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    p.add_argument("--repeats", type=int, default=3)
    args = p.parse_args()
    sys.path.insert(0, args.reference)
    sys.path.insert(0, ROOT)
    from stepquant.core import delta_step
    from stepquant.quantization import QuantizationPlan, StateCodec
    from oracle import stepquant_oracle as O

    torch.set_num_threads(args.threads)
    heads, qk, dim, batch = 32, 16, 128, args.requests
    rng = np.random.default_rng(1)
    widths = np.array([4] * 8 + [6] * 16 + [8] * 8)
    rng.shuffle(widths)
    bits = np.repeat(widths[:, None], dim, 1)
    impact = (rng.random((heads, dim)) + 0.5).astype(np.float32)
    state = (rng.standard_normal((batch, heads, dim, dim)) * 0.1).astype(np.float32)
    q = rng.standard_normal((batch, qk, dim)).astype(np.float32)
    k = rng.standard_normal((batch, qk, dim)).astype(np.float32)
    v = rng.standard_normal((batch, heads, dim)).astype(np.float32)
    a = rng.standard_normal((batch, heads)).astype(np.float32)
    b = rng.standard_normal((batch, heads)).astype(np.float32)
    a_log = (rng.random(heads) * math.log(16)).astype(np.float32)
    dt_bias = np.zeros(heads, np.float32)

    # reference torch path
    plan = QuantizationPlan("gdn", torch.from_numpy(bits), torch.from_numpy(impact))
    codec = StateCodec(plan)
    packed = codec.encode(torch.from_numpy(state))
    tq, tk = torch.from_numpy(q), torch.from_numpy(k)

    def reference_step(packed):
        s = codec.decode(packed)
        qn = tq * torch.rsqrt(tq.square().sum(-1, keepdim=True) + 1e-6) * dim ** -0.5
        kn = tk * torch.rsqrt(tk.square().sum(-1, keepdim=True) + 1e-6)
        qn, kn = qn.repeat_interleave(heads // qk, 1), kn.repeat_interleave(heads // qk, 1)
        g = -torch.from_numpy(a_log).exp() * torch.nn.functional.softplus(torch.from_numpy(a + dt_bias))
        _, s = delta_step(s, qn, kn, torch.from_numpy(v), g, torch.from_numpy(b).sigmoid())
        return codec.encode(s)

    # numpy port (the benchmark's CPU baseline on the GPU box)
    oplan = O.Plan("gdn", bits, impact)
    opacked = O.codec_encode(state, oplan)

    def port_step(packed):
        s = O.codec_decode(packed, oplan)
        qp, kp, g, beta = O.prepare_inputs(q, k, a, b, heads, kda=False, normalize=True, scale=dim ** -0.5,
                                           a_log=a_log, dt_bias=dt_bias)
        _, s = O.delta_step(s, qp, kp, v, g, beta)
        return O.codec_encode(s, oplan)

    def best(fn, packed):
        times = []
        for _ in range(args.repeats):
            t0 = time.perf_counter()
            packed = fn(packed)
            times.append(time.perf_counter() - t0)
        return min(times)

    t_ref = best(reference_step, packed)
    t_port = best(port_step, opacked)
    updates = batch * heads
    print(json.dumps({"requests": batch, "heads": heads, "torch_threads": args.threads,
                      "reference_torch_s_per_update": t_ref / updates, "numpy_port_s_per_update": t_port / updates,
                      "port_over_reference_time": t_port / t_ref}))


if __name__ == "__main__":
    main()
