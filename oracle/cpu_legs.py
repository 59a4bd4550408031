"""CPU baselines of the hot path, timed on the host cores.

TEST INFRASTRUCTURE ONLY: bench.py runs this as its CPU legs (in a separate
process, so that torch's thread pool is configured before torch loads).

    OMP_WAIT_POLICY=PASSIVE python -m oracle.cpu_legs [--seconds S] [--steps K --warmup W]

Legs (seeded synthetic inputs of the benchmark configurations):
  router        the reference's router op chain (oracle/aten_chain.py) on the
                full 65536 x 256 batch: K timed steps after W warm-ups
                when --steps is given, else as many as fit in the time bound
  router_fused  the oracle's C restatement of the same router (OpenMP)
  silu_and_mul  the chain on a row sample of x bf16 [8192, 2 x 18432]
  rms_norm      the chain on a row sample of x bf16 [8192, 7168]
  gated_mlp     the TP=1 gated MLP H=4096 / I=14336 step on a token sample

Prints one JSON object.  The reference's raw sigmoid / silu loops are single
threaded (they run on one worker thread of its launch queue); the ATen ops
use torch's intra-op threads.  OMP_WAIT_POLICY=PASSIVE keeps those threads
from spinning while the single-threaded loops run.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _host():
    model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    import torch

    return {"nproc": os.cpu_count(), "cpu_model": model, "torch_threads": torch.get_num_threads(),
            "omp_wait_policy": os.environ.get("OMP_WAIT_POLICY", "")}


def _time(fn, seconds, min_runs=3, max_runs=200, warmup=1):
    for _ in range(warmup):
        fn()
    times = []
    end = time.perf_counter() + seconds
    while len(times) < min_runs or (time.perf_counter() < end and len(times) < max_runs):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def router_leg(seconds, steps=None, warmup=None):
    import configs as C
    from oracle import aten_chain

    T = 65536
    g, b = C.router_inputs(C.deepseek_v3(T))

    def run():
        aten_chain.grouped_topk_chain(g, 8, True, 8, 4, "sigmoid", 2.5, b)

    if steps is not None:
        for _ in range(warmup or 0):
            run()
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
        med, n = statistics.median(times), len(times)
    else:
        med, n = _time(run, seconds)
    return {"value": round(T / med / 1e6, 4), "unit": "Mtok/s", "ms_per_batch": round(med * 1e3, 2),
            "runs": n, "sample": f"{n} runs of the full {T}x256 batch through the reference's op chain "
                                 "(raw sigmoid loop on one thread, ATen CPU ops on the intra-op threads)"}


def router_fused_leg(seconds):
    import configs as C
    import oracle

    T = 65536
    g, b = C.router_inputs(C.deepseek_v3(T))
    gn, bn = g.numpy(), b.numpy()
    threads = os.cpu_count() or 1
    med, n = _time(lambda: oracle.grouped_topk(gn, 8, True, 8, 4, "sigmoid", 2.5, bn, nthreads=threads), seconds)
    return {"value": round(T / med / 1e6, 4), "unit": "Mtok/s", "ms_per_batch": round(med * 1e3, 2), "runs": n,
            "threads": threads, "sample": f"{n} runs of the full batch, the oracle's fused C restatement"}


def silu_leg(seconds, rows=256):
    import configs as C
    from oracle import aten_chain

    d = 18432
    x = C.silu_inputs(rows, d)
    med, n = _time(lambda: aten_chain.silu_and_mul_chain(x), seconds)
    nbytes = rows * 2 * d * 2 + rows * d * 2
    return {"us_per_full_call": round(med * 8192 / rows * 1e6, 1), "gbs": round(nbytes / med / 1e9, 3),
            "runs": n, "sample": f"{rows} of 8192 rows of x bf16 [8192, {2 * d}] per run, scaled to the full call"}


def rms_leg(seconds, rows=1024):
    import configs as C
    from oracle import aten_chain

    H = 7168
    x, w = C.rms_inputs(rows, H)
    med, n = _time(lambda: aten_chain.rms_norm_chain(x, w, C.RMS_EPS), seconds)
    nbytes = 2 * rows * H * 2 + H * 2
    return {"us_per_full_call": round(med * 8192 / rows * 1e6, 1), "gbs": round(nbytes / med / 1e9, 3),
            "runs": n, "sample": f"{rows} of 8192 rows of x bf16 [8192, {H}] per run, scaled to the full call"}


def mlp_leg(seconds, tokens=256):
    import torch

    import configs as C
    from oracle import aten_chain

    cfg = C.MLP_M1
    x, _, wgu, wd = C.mlp_weights(cfg, 1, 0)
    xs = x[:tokens].contiguous()
    med, n = _time(lambda: aten_chain.gated_mlp_chain(xs, wgu, wd), seconds, min_runs=2)
    flops = 2 * tokens * cfg.H * cfg.I * 3
    del torch
    return {"tflops": round(flops / med / 1e12, 4), "ms_per_full_step": round(med * cfg.T / tokens * 1e3, 1),
            "runs": n, "sample": f"{tokens} of {cfg.T} tokens of the H={cfg.H} I={cfg.I} step per run (TP=1), "
                                 "scaled to the full step"}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seconds", type=float, default=8.0, help="time bound of each leg")
    ap.add_argument("--steps", type=int, default=None, help="exact router steps (reference arm)")
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--legs", default="router,router_fused,silu_and_mul,rms_norm,gated_mlp")
    a = ap.parse_args(argv)
    sys.path.insert(0, os.path.join(_ROOT, "tests", "golden"))
    sys.path.insert(0, _ROOT)
    legs = set(a.legs.split(","))
    out = {"host": _host()}
    if "router" in legs:
        out["router"] = router_leg(a.seconds, a.steps, a.warmup)
    if "router_fused" in legs:
        out["router_fused"] = router_fused_leg(a.seconds)
    if "silu_and_mul" in legs:
        out["silu_and_mul"] = silu_leg(a.seconds)
    if "rms_norm" in legs:
        out["rms_norm"] = rms_leg(a.seconds)
    if "gated_mlp" in legs:
        out["gated_mlp"] = mlp_leg(a.seconds)
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
