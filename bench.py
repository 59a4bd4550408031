"""Benchmark of the mcpu device hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): the DeepSeek-V3-style grouped_topk router over one
batch of 65536 tokens x 256 experts (fp32 logits N(0,1), fp32 bias N(0,0.01),
8 groups, top-4 groups, top-8, sigmoid + bias, renormalised, x2.5).  Inputs
rotate through 8 device buffers (8 x 67 MB > 2 x L2) so no step reads its
logits from L2.  Steps are replayed from a CUDA graph of the C-ABI launches;
W warm-up steps, then K timed steps between barriers and device syncs,
timed with CUDA events on the launching stream, max over ranks.

Multi-GPU: the router is independent per token, so N ranks run N replicas
(weak scaling, no collective on the data path); `value` is all ranks'
tokens over the slowest rank's time.  The "tp_mlp" object reports the other
half of the metric: the gated MLP H=4096 / I=14336 / T=2048 in bf16,
tensor-parallel over the N ranks (TP=N), through the mcpu device (tcgen05
GEMMs, fused SwiGLU) and its NCCL ProcessGroup (SUM all-reduce), in whole-job
TFLOP/s over the slowest rank.

--impl reference times the reference algorithm on the host cores (the
oracle's C restatement of the reference's CPU path, all threads), rank 0
only, on the same configuration.

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

METRIC = "grouped_topk Mtok/s + HBM GB/s; TP-MLP TFLOP/s at 1/2/4/8 B200 vs CPU"
T, E, G, TG, K = 65536, 256, 8, 4, 8
BYTES_PER_TOKEN = E * 4 + K * 4 + K * 4  # logits in, weights + ids out
N_BUFFERS = 8
GRAPH_STEPS = 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="bound on the host-core baseline's sampling time")
    ap.add_argument("--legs", default="e2e,bw,moe,sampler,mlp,cpu",
                    help="extra legs besides the router timing (comma list of e2e, bw, moe, sampler, mlp, cpu; "
                         "'none' for the router alone, e.g. under a profiler)")
    a = ap.parse_args()
    a.legs = set() if a.legs == "none" else set(a.legs.split(","))
    return a


def workload_config(n):
    return {
        "workload": f"grouped_topk T={T} E={E} G={G} topk_group={TG} topk={K} sigmoid+bias "
                    "renormalize x2.5 (DeepSeek-V3 router)",
        "tokens_per_step_per_gpu": T,
        "global_batch": T * n,
        "l2": f"inputs rotate over {N_BUFFERS} device buffers of {T * E * 4 / 1e6:.1f} MB "
              "(> 2 x L2), no L2 flush needed",
        "parallelism": f"replicas x{n}",
    }


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(name: str):
    """DRAM bytes per launch recorded from an ncu capture in profiles/."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.reasons = 0
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
            return self
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.reasons |= int(r) & ~0x1
            except Exception:
                pass
            time.sleep(0.005)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {
            "sm_mhz": statistics.median(self.samples) if self.samples else None,
            "sm_max_mhz": self.max_mhz,
            "samples": len(self.samples),
            "reasons": [n for b, n in self.REASONS.items() if self.reasons & b],
            "source": "nvml, 5 ms polling during the timed region",
        }


# ---------------------------------------------------------------- CPU leg
def cpu_baseline(seconds: float):
    """The reference algorithm on the host cores: the oracle's C restatement
    of the reference's CPU path (kind "port"), all host threads."""
    import numpy as np

    import configs as C
    import oracle

    cfg = C.deepseek_v3(T)
    gating, bias = C.router_inputs(cfg)
    g, b = gating.numpy(), bias.numpy()
    threads = os.cpu_count() or 1
    oracle.grouped_topk(g[:1024], K, True, G, TG, "sigmoid", 2.5, b, nthreads=threads)
    times = []
    t_end = time.perf_counter() + seconds
    while True:
        t0 = time.perf_counter()
        oracle.grouped_topk(g, K, True, G, TG, "sigmoid", 2.5, b, nthreads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 200:
            break
    med = statistics.median(times)
    return {
        "value": round(T / med / 1e6, 4),
        "unit": "Mtok/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{len(times)} runs of the full {T}x{E} batch (median {med * 1e3:.1f} ms), "
                  f"oracle C restatement with glibc expf, {threads} OpenMP threads",
    }


# ---------------------------------------------------------------- dist
def dist_setup(n):
    import torch

    import torch_mcpu_b200.device  # noqa: F401  the mcpu device + its NCCL ProcessGroup

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    torch.mcpu.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # the reference's init string: gloo for CPU tensors, the mcpu backend
        # (NCCL over NVLink here) for mcpu tensors
        dist.init_process_group("cpu:gloo,mcpu:mcpu", timeout=datetime.timedelta(seconds=120))
        pg = dist
    return rank, world, local, pg


def barrier(pg):
    if pg is not None:
        pg.barrier()


def max_over_ranks(pg, v: float, dev=None) -> float:
    if pg is None:
        return v
    import torch

    t = torch.tensor([v], dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- TP MLP
def _graph_ms(step, pg, steps, warmup):
    """Captures `step` once in a CUDA graph on a side stream and returns the
    slowest rank's mean CUDA-event time of `steps` replays (ms)."""
    import torch

    side = torch.mcpu.Stream()
    graph = torch.mcpu.Graph()
    with torch.mcpu.stream(side):
        for _ in range(max(3, warmup)):
            step()
        side.synchronize()
        barrier(pg)
        with graph.capture():
            step()
        side.synchronize()
        barrier(pg)
        for _ in range(3):
            graph.replay()
        side.synchronize()
        barrier(pg)
        e0 = torch.Event(device="mcpu", enable_timing=True)
        e1 = torch.Event(device="mcpu", enable_timing=True)
        e0.record(side)
        for _ in range(steps):
            graph.replay()
        e1.record(side)
        e1.synchronize()
    graph.reset()
    return max_over_ranks(pg, e0.elapsed_time(e1)) / steps


def tp_mlp_leg(rank, world, pg, steps, warmup):
    """Gated MLP H=4096, I=14336, T=2048 (bf16), tensor-parallel over the
    N ranks: fused gate/up GEMM + SwiGLU, then the row-parallel down
    projection and the SUM all-reduce of the partials — at N > 1 as one
    kernel over NVLink (mm_allreduce in a symmetric window), with the
    mm + NCCL all-reduce form timed beside it.  Whole-job TFLOP/s over the
    slowest rank's CUDA-event time."""
    import torch

    import configs as C

    cfg = C.MLP_M1
    x, _, wgu, wd = C.mlp_weights(cfg, world, rank)
    from torch_mcpu_b200 import ops, symm

    xm = x.to("mcpu")
    wgu_il = ops.interleave_gate_up(wgu).to("mcpu")
    wdm = wd.to("mcpu")
    act = torch.empty(cfg.T, wgu.size(0) // 2, dtype=torch.bfloat16, device="mcpu")
    y = torch.empty(cfg.T, cfg.H, dtype=torch.bfloat16, device="mcpu")

    def step_nccl():
        torch.ops.mcpu.gemm_swiglu.out(xm, wgu_il, out=act)
        torch.mm(act, wdm.t(), out=y)
        if pg is not None:
            pg.all_reduce(y)

    nccl_ms = _graph_ms(step_nccl, pg, steps, warmup)
    ms, mode = nccl_ms, "mm + all_reduce over the mcpu ProcessGroup (NCCL)" if world > 1 else "mm"
    if world > 1:
        win = symm.SymmetricWindow(symm.window_bytes(cfg.T, cfg.H, world))

        def step_fused():
            torch.ops.mcpu.gemm_swiglu.out(xm, wgu_il, out=act)
            symm.mm_allreduce(act, wdm, win)

        ms = _graph_ms(step_fused, pg, steps, warmup)
        mode = "down projection + all-reduce fused over NVLink (mm_allreduce, symmetric window)"
        torch.mcpu.synchronize()
        if ops.device_error():
            raise RuntimeError("mm_allreduce: a bounded wait ran out during the TP leg")
        win.close()
    flops = 2 * cfg.T * cfg.H * cfg.I * 3
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        peaks = {"bf16_tflops": pk["bf16_tflops"], "bf16_tflops_sustained": pk["bf16_tflops_sustained"]}
    except Exception:
        peaks = {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "kind": "fallback"}
    whole = flops / (ms * 1e-3) / 1e12
    per_gpu = whole / world
    return {
        "config": f"gated MLP bf16 H={cfg.H} I={cfg.I} T={cfg.T} TP={world} (gate/up column-parallel, "
                  f"down row-parallel; {mode}; step replayed from a CUDA graph)",
        "nccl_ms_per_step": round(nccl_ms, 4),
        "tflops": round(whole, 1),
        "per_gpu_tflops": round(per_gpu, 1),
        "ms_per_step": round(ms, 4),
        "frac_of_bf16_peak": round(per_gpu / peaks["bf16_tflops"], 4),
        "frac_of_bf16_sustained": round(per_gpu / peaks["bf16_tflops_sustained"], 4),
        "steps": steps,
        "flops_per_step": flops,
    }


def bandwidth_leg(dev, reps=20):
    """silu_and_mul on [8192, 2 x 18432] and rms_norm on [8192, 7168] (bf16,
    DeepSeek-V3 dense-MLP intermediate and hidden widths): CUDA-event time
    per call over rotating inputs
    larger than L2, achieved GB/s of the algorithmic bytes."""
    import torch

    from torch_mcpu_b200 import ops

    peak, peak_kind = measured_peaks()
    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    T1, d = 8192, 18432
    xs = [torch.randn(T1, 2 * d, generator=g, device=dev).to(torch.bfloat16) for _ in range(2)]
    o = torch.empty(T1, d, dtype=torch.bfloat16, device=dev)
    T2, H = 8192, 7168
    xr = [torch.randn(T2, H, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
    wr = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(torch.bfloat16)
    o2 = torch.empty(T2, H, dtype=torch.bfloat16, device=dev)
    cases = [
        ("silu_and_mul", f"x bf16 [{T1}, {2 * d}] -> [{T1}, {d}]", T1 * 2 * d * 2 + T1 * d * 2,
         lambda i: ops.silu_and_mul(o, xs[i % 2])),
        ("rms_norm", f"x bf16 [{T2}, {H}], w [{H}], eps 1e-6", 2 * T2 * H * 2 + H * 2,
         lambda i: ops.rms_norm(o2, xr[i % 3], wr, 1e-6)),
    ]
    for name, shape, nbytes, fn in cases:
        for i in range(3):
            fn(i)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"shape": shape, "us_per_call": round(us, 2), "algorithmic_bytes": nbytes,
                     "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "frac": round(gbs / peak, 4),
                     "peak_kind": peak_kind}
    return out


def moe_leg(dev, ids, stream, reps=8, per_graph=32):
    """MoE dispatch after the router: moe_align_block_size on the router's
    own topk_ids [65536, 8] (256 experts, block 64), replayed from a CUDA
    graph; time per call and GB/s of its algorithmic bytes (ids read once,
    sorted ids and block experts written once)."""
    import ctypes

    import torch

    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    peak, peak_kind = measured_peaks()
    numel, E_, bs = ids.numel(), 256, 64
    cap = min(numel + E_ * (bs - 1), numel * bs)
    nblk = -(-cap // bs)
    srt = torch.empty(cap, dtype=torch.int32, device=dev)
    eid = torch.empty(nblk, dtype=torch.int32, device=dev)
    npad = torch.empty(1, dtype=torch.int32, device=dev)
    wsb = ctypes.c_uint64()
    _lib.check(lib.mcpu_moe_align_workspace_bytes(numel, E_, ctypes.byref(wsb)), "moe workspace")
    work = torch.empty(wsb.value, dtype=torch.uint8, device=dev)

    def call():
        _lib.check(lib.mcpu_moe_align_block_size(ids.data_ptr(), numel, E_, bs, srt.data_ptr(), cap, eid.data_ptr(),
                                                 nblk, npad.data_ptr(), work.data_ptr(), wsb.value,
                                                 stream.cuda_stream), "moe_align_block_size")

    with torch.cuda.stream(stream):
        for _ in range(3):
            call()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(per_graph):
            call()
    with torch.cuda.stream(stream):
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * per_graph)
    del graph
    nbytes = numel * 4 + cap * 4 + nblk * 4 + 4
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"shape": f"topk_ids int32 [{numel // 8}, 8] from the router, {E_} experts, block {bs}",
            "us_per_call": round(us, 2), "launches_per_call": 2, "algorithmic_bytes": nbytes,
            "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "frac": round(gbs / peak, 4), "peak_kind": peak_kind}


def sampler_leg(dev, reps=20):
    """The reference's vLLM sampler ops on a decode batch: 256 rows x 128256
    vocab fp32 logits (131 MB, more than L2): min_p in place (p = 0.05 on
    every row), top-5 log-probabilities and the repetition / frequency /
    presence penalties in place; CUDA-event time per call and
    GB/s of the algorithmic bytes (the logits read once; each row's second
    pass re-reads it from L2)."""
    import torch

    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    peak, peak_kind = measured_peaks()
    rows, vocab = 256, 128256
    g = torch.Generator(device=dev).manual_seed(9)
    xs = [3.0 * torch.randn(rows, vocab, generator=g, device=dev) for _ in range(2)]
    idx = torch.arange(rows, dtype=torch.int32, device=dev)
    mp = torch.full((rows,), 0.05, dtype=torch.float32, device=dev)
    ids = torch.randint(0, vocab, (rows, 5), device=dev, generator=g)
    out = torch.empty(rows, 5, dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream(dev).cuda_stream
    cases = [
        ("vllm_min_p", rows * vocab * 4,
         lambda i: _lib.check(lib.mcpu_vllm_min_p(xs[i % 2].data_ptr(), 0, rows, vocab, idx.data_ptr(),
                                                  mp.data_ptr(), vocab, s), "min_p")),
        ("vllm_topk_log_softmax", rows * vocab * 4,
         lambda i: _lib.check(lib.mcpu_vllm_topk_log_softmax(out.data_ptr(), xs[i % 2].data_ptr(), 0, rows, vocab,
                                                             ids.data_ptr(), 5, 5, vocab, s), "log_softmax")),
    ]
    # penalties: every row its own request, repetition 1.1, frequency and
    # presence 0.1, prompt bits and output counts random; bytes = the logits
    # read and written, the counts and the bit mask read once
    cols = (vocab + 31) // 32
    rep = torch.full((rows,), 1.1, dtype=torch.float32, device=dev)
    fp = torch.full((rows,), 0.1, dtype=torch.float32, device=dev)
    pbm = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, cols), dtype=torch.int32, device=dev, generator=g)
    obc = torch.randint(0, 3, (rows, vocab), dtype=torch.int32, device=dev, generator=g)
    zeros = torch.zeros(rows, dtype=torch.int32, device=dev)
    cases.append(
        ("vllm_penalties", rows * vocab * 12 + rows * cols * 4,
         lambda i: _lib.check(lib.mcpu_vllm_penalties(xs[i % 2].data_ptr(), 0, rows, vocab, idx.data_ptr(),
                                                      zeros.data_ptr(), zeros.data_ptr(), rep.data_ptr(),
                                                      fp.data_ptr(), fp.data_ptr(), rows, pbm.data_ptr(), cols,
                                                      obc.data_ptr(), vocab, vocab, 0, s), "penalties")))
    res = {}
    for name, nbytes, fn in cases:
        for i in range(3):
            fn(i)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            fn(i)
        e1.record()
        e1.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        gbs = nbytes / (us * 1e-6) / 1e9
        res[name] = {"shape": f"logits fp32 [{rows}, {vocab}]", "us_per_call": round(us, 2),
                     "algorithmic_bytes": nbytes, "achieved_gbs": round(gbs, 1), "peak_gbs": peak,
                     "frac": round(gbs / peak, 4), "peak_kind": peak_kind}
    return res


# ---------------------------------------------------------------- ours
def run_ours(a):
    import numpy as np
    import torch

    import configs as C
    from torch_mcpu_b200 import _lib

    rank, world, local, pg = dist_setup(a.gpus)
    dev = torch.device("cuda", local)
    lib = _lib.load()

    cfg = C.deepseek_v3(T)
    gating_cpu, bias_cpu = C.router_inputs(cfg)
    bufs = [gating_cpu.to(dev)]
    for i in range(1, N_BUFFERS):  # distinct contents, same distribution
        g = torch.Generator(device=dev).manual_seed(100 + i)
        bufs.append(torch.randn(T, E, generator=g, device=dev))
    bias = bias_cpu.to(dev)
    w = torch.empty(T, K, dtype=torch.float32, device=dev)
    ids = torch.empty(T, K, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(dev)

    def launch(i):
        rc = lib.mcpu_grouped_topk(bufs[i % N_BUFFERS].data_ptr(), 0, T, E, G, TG, K, 1, 2.5,
                                   bias.data_ptr(), 1, w.data_ptr(), ids.data_ptr(),
                                   stream.cuda_stream)
        if rc != 0:
            _lib.check(rc, "grouped_topk")

    # correctness spot check of this exact configuration before timing
    with torch.cuda.stream(stream):
        launch(0)
    stream.synchronize()
    if rank == 0:
        import oracle

        ow, oids, _, _ = oracle.grouped_topk(gating_cpu[:4096].numpy(), K, True, G, TG, "sigmoid",
                                             2.5, bias_cpu.numpy(), exp_mode=oracle.EXP_CR)
        got = np.sort(ids[:4096].cpu().numpy(), 1)
        if not np.array_equal(got, np.sort(oids, 1)):
            raise SystemExit("bench: router output differs from the oracle; refusing to time it")

    # CUDA graph of GRAPH_STEPS launches (rotating buffers)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for i in range(3):
            launch(i)
    stream.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(GRAPH_STEPS):
            launch(i)
    reps_w = max(1, -(-a.warmup // GRAPH_STEPS))
    reps = max(1, -(-a.steps // GRAPH_STEPS))
    steps = reps * GRAPH_STEPS

    exact_before = ctypes.c_ulonglong(0)
    lib.mcpu_grouped_topk_exact_rows(ctypes.byref(exact_before), 1)
    with torch.cuda.stream(stream):
        for _ in range(reps_w):
            graph.replay()
    stream.synchronize()
    barrier(pg)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(reps):
                graph.replay()
            ev1.record(stream)
        ev1.synchronize()
    torch.cuda.synchronize(dev)
    barrier(pg)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(pg, ms)
    exact = ctypes.c_ulonglong(0)
    lib.mcpu_grouped_topk_exact_rows(ctypes.byref(exact), 0)
    exact_per_step = exact.value / (steps + reps_w * GRAPH_STEPS)

    # e2e through the C-ABI with host buffers: every step copies its logits
    # host -> device, routes them and copies its weights and ids back.  Two
    # sets of device buffers and three streams let step i+1's input copy and
    # step i-1's result copy run while step i's router runs.
    host_in = torch.empty(T, E, dtype=torch.float32, pin_memory=True)
    host_in.copy_(gating_cpu)
    host_w = [torch.empty(T, K, dtype=torch.float32, pin_memory=True) for _ in range(2)]
    host_ids = [torch.empty(T, K, dtype=torch.int32, pin_memory=True) for _ in range(2)]
    dbufs = [bufs[0], bufs[1]]
    w2 = [w, torch.empty_like(w)]
    ids2 = [ids, torch.empty_like(ids)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    loaded = [torch.cuda.Event() for _ in range(2)]
    routed = [torch.cuda.Event() for _ in range(2)]
    returned = [torch.cuda.Event() for _ in range(2)]
    used = [False, False]
    h2d = T * E * 4
    d2h = T * K * 8

    def e2e_step(i):
        b = i % 2
        if used[b]:
            s_in.wait_event(routed[b])  # the router that last read this set is done
        _lib.check(lib.orMemcpyAsync(dbufs[b].data_ptr(), host_in.data_ptr(), h2d, 1, s_in.cuda_stream), "H2D")
        loaded[b].record(s_in)
        stream.wait_event(loaded[b])
        if used[b]:
            stream.wait_event(returned[b])  # this set's last results are back on the host
        _lib.check(lib.mcpu_grouped_topk(dbufs[b].data_ptr(), 0, T, E, G, TG, K, 1, 2.5,
                                         bias.data_ptr(), 1, w2[b].data_ptr(), ids2[b].data_ptr(),
                                         stream.cuda_stream), "grouped_topk")
        routed[b].record(stream)
        s_out.wait_event(routed[b])
        _lib.check(lib.orMemcpyAsync(host_w[b].data_ptr(), w2[b].data_ptr(), T * K * 4, 2, s_out.cuda_stream), "D2H")
        _lib.check(lib.orMemcpyAsync(host_ids[b].data_ptr(), ids2[b].data_ptr(), T * K * 4, 2, s_out.cuda_stream),
                   "D2H")
        returned[b].record(s_out)
        used[b] = True

    e2e_ms = None
    if "e2e" in a.legs:
        e2e_steps = max(3, min(a.steps, 200))
        for i in range(4):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        barrier(pg)
        ev0.record(s_in)
        for i in range(e2e_steps):
            e2e_step(i)
        ev1.record(s_out)
        ev1.synchronize()
        torch.cuda.synchronize(dev)
        barrier(pg)
        e2e_ms = max_over_ranks(pg, ev0.elapsed_time(ev1)) / e2e_steps
    del graph
    bw = bandwidth_leg(dev) if "bw" in a.legs else None
    moe = moe_leg(dev, ids, stream) if "moe" in a.legs else None
    sampler = sampler_leg(dev) if "sampler" in a.legs else None
    mlp = tp_mlp_leg(rank, world, pg, steps=max(10, min(a.steps, 50)), warmup=3) if "mlp" in a.legs else None

    if rank == 0:
        per_step = ms_max / steps
        peak, peak_kind = measured_peaks()
        achieved = BYTES_PER_TOKEN * T / (per_step * 1e-3) / 1e9
        traffic = profiled_traffic("grouped_topk_T65536_E256.md")
        line = {
            "metric": METRIC,
            "value": round(T * world / (per_step * 1e-3) / 1e6, 2),
            "unit": "Mtok/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": reps_w * GRAPH_STEPS,
            "ms_per_step": round(per_step, 6),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded N(0,1) logits, N(0,0.01) bias)",
            "config": workload_config(world),
            "roofline": {
                "bound": "hbm",
                "achieved": round(achieved, 1),
                "peak": peak,
                "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "peak_kind": peak_kind,
                "traffic": traffic,
                "algorithmic_bytes_per_launch": BYTES_PER_TOKEN * T,
            },
            "e2e": None if e2e_ms is None else {
                "value": round(T * world / (e2e_ms * 1e-3) / 1e6, 2),
                "unit": "Mtok/s",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": "per step: orMemcpyAsync H2D (pinned) -> mcpu_grouped_topk -> orMemcpyAsync D2H (pinned); "
                        "two buffer sets on copy-in / router / copy-out streams, so step i+1's input copy "
                        "overlaps step i's router",
            },
            "clocks": clk.summary(),
            "gpu_launches": steps,
            "exact_path_rows_per_step": round(exact_per_step, 2),
            "bandwidth_ops": bw,
            "moe_dispatch": moe,
            "sampler_ops": sampler,
            "tp_mlp": mlp,
        }
        line["cpu_baseline"] = cpu_baseline(a.cpu_seconds) if (world == 1 and "cpu" in a.legs) else None
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    base = cpu_baseline(a.cpu_seconds)
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": base["value"],
        "unit": "Mtok/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(T / (base["value"] * 1e6) * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) logits, N(0,0.01) bias)",
        "config": workload_config(1),
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "Mtok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
