"""Benchmark of the mcpu device hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): the DeepSeek-V3-style grouped_topk router over one
batch of 65536 tokens x 256 experts (fp32 logits N(0,1), fp32 bias N(0,0.01),
8 groups, top-4 groups, top-8, sigmoid + bias, renormalised, x2.5).  Inputs
rotate through 8 device buffers (8 x 67 MB > 2 x L2) so no step reads its
logits from L2.  W warm-up launches, then exactly K timed launches replayed
from CUDA graphs of the C-ABI call, between barriers and device syncs, timed
with CUDA events on the launching stream, max over ranks.

Multi-GPU: the router is independent per token, so N ranks run N replicas
(weak scaling, no collective on the data path); `value` is all ranks'
tokens over the slowest rank's time.  The "tp_mlp" object reports the other
half of the metric: the gated MLP of the TP example (H=4096 / I=14336 /
T=2048) and the pre-rms_norm SwiGLU block (H=7168 / I=18432, T=8192 and
T=256) in bf16, tensor-parallel over the N ranks (TP=N), through the mcpu
device (tcgen05 GEMMs, fused SwiGLU) with the down projection and the SUM
all-reduce fused over NVLink, the mm + NCCL form timed beside it; each case
carries its TP=1 time on rank 0 of the same job and the scaling efficiency
t_TP1 / (N t_N), and at N > 1 the fused all-reduce is checked bit for bit
against the fp32 sum in rank order of the gathered partials (a mismatch
fails the run).

--impl reference times the reference's path on the host cores, rank 0
only, on the same configuration: its router op chain (the ATen CPU kernels
its mcpu ops run, in its order, with its single-threaded raw sigmoid loop)
over the full batch per step, with silu_and_mul, rms_norm and the gated
MLP step timed beside it (oracle/cpu_legs.py).

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
    ap.add_argument("--steps", type=int, default=640)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=6.0,
                    help="bound on the host-core baseline's sampling time")
    ap.add_argument("--legs", default="e2e,sweep,bw,moe,sampler,mlp,cpu",
                    help="extra legs besides the router timing (comma list of e2e, sweep, bw, moe, sampler, mlp, "
                         "cpu; 'none' for the router alone, e.g. under a profiler)")
    ap.add_argument("--mlp-cases", default="M1,M2_T8192,M2_T256",
                    help="tensor-parallel MLP cases of the mlp leg (comma list of M1, M2_T8192, M2_T256)")
    a = ap.parse_args()
    if a.steps < 1 or a.warmup < 0:
        ap.error("--steps must be >= 1 and --warmup >= 0")
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
    """Samples the SM clock and the clock-event reasons through NVML, every
    5 ms from __enter__ to __exit__, with the time of each sample so that a
    summary can be given for a window (e.g. one timed region) as well as for
    the whole device-busy span."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int):
        self.index = index
        self.samples = []  # (monotonic time, SM MHz, reason bits)
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
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self._h)
                self.samples.append((time.monotonic(), mhz, int(r) & ~0x1))
            except Exception:
                pass
            time.sleep(0.005)

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self, windows=None, what="the timed regions"):
        sel = self.samples
        if windows:
            sel = [s for s in self.samples if any(a <= s[0] <= b for a, b in windows)]
        reasons = 0
        for s in sel:
            reasons |= s[2]
        return {
            "sm_mhz": statistics.median(s[1] for s in sel) if sel else None,
            "sm_max_mhz": self.max_mhz,
            "samples": len(sel),
            "reasons": [n for b, n in self.REASONS.items() if reasons & b],
            "source": f"nvml, 5 ms polling during {what}",
        }


# ---------------------------------------------------------------- CPU leg
def cpu_legs(seconds: float, steps=None, warmup=None, legs=None):
    """The reference's path on the host cores (oracle/cpu_legs.py), in a
    child process so that torch's intra-op threads are configured (passive
    OpenMP waits) before torch loads."""
    import subprocess

    env = dict(os.environ)
    env.setdefault("OMP_WAIT_POLICY", "PASSIVE")
    env.pop("CUDA_VISIBLE_DEVICES", None)
    cmd = [sys.executable, "-m", "oracle.cpu_legs", "--seconds", str(seconds)]
    if steps is not None:
        cmd += ["--steps", str(steps), "--warmup", str(warmup or 0)]
    if legs:
        cmd += ["--legs", legs]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    if r.returncode != 0:
        raise SystemExit(f"bench: CPU legs failed:\n{r.stderr[-2000:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def cpu_baseline(seconds: float):
    """cpu_baseline of the line: the reference's router op chain on the full
    batch (kind "port": a restatement of its mcpu path, the same ATen CPU
    kernels in the same order with its single-threaded raw sigmoid loop),
    with the other legs of the path beside it."""
    legs = cpu_legs(seconds)
    r = legs["router"]
    return {
        "value": r["value"],
        "unit": "Mtok/s",
        "cores": legs["host"]["torch_threads"],
        "kind": "port",
        "sample": r["sample"] + f"; host: {legs['host']['nproc']} x {legs['host']['cpu_model']}",
        "legs": legs,
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


def _bf16_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        return {"bf16_tflops": pk["bf16_tflops"], "bf16_tflops_sustained": pk["bf16_tflops_sustained"],
                "kind": "measured"}
    except Exception:
        return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "kind": "fallback"}


MLP_CASES = {"M1": "MLP_M1", "M2_T8192": "MLP_M2_LARGE", "M2_T256": "MLP_M2_SMALL"}


class _Shard:
    """One rank's weights and buffers of a TP MLP case on the mcpu device."""

    def __init__(self, cfg, tp, rank):
        import torch

        import configs as C
        from torch_mcpu_b200 import ops

        x, rms_w, wgu, wd = C.mlp_weights(cfg, tp, rank)
        self.cfg = cfg
        self.x = x.to("mcpu")
        self.rms = None if rms_w is None else rms_w.to("mcpu")
        self.wgu = ops.interleave_gate_up(wgu).to("mcpu")
        self.wd = wd.to("mcpu")
        self.normed = torch.empty(cfg.T, cfg.H, dtype=torch.bfloat16, device="mcpu") if cfg.pre_norm else None
        self.act = torch.empty(cfg.T, wgu.size(0) // 2, dtype=torch.bfloat16, device="mcpu")
        self.y = torch.empty(cfg.T, cfg.H, dtype=torch.bfloat16, device="mcpu")

    def front(self):
        """rms_norm (replicated) and the column-parallel gate/up GEMM + SwiGLU."""
        import torch

        import configs as C

        h = self.x
        if self.rms is not None:
            torch.ops.mcpu.rms_norm(self.normed, self.x, self.rms, C.RMS_EPS)
            h = self.normed
        torch.ops.mcpu.gemm_swiglu.out(h, self.wgu, out=self.act)

    def partial(self):
        import torch

        torch.mm(self.act, self.wd.t(), out=self.y)
        return self.y


def _check_fused(shard, win, world, pg):
    """The fused down projection + all-reduce against the fp32 sum, in rank
    order, of every rank's bf16 partial (gathered with NCCL), rounded once
    to bf16: bit for bit on rank 0, and the same bits on every rank (digest
    of each rank's output).  The NCCL all-reduce of the same partials is
    compared too (its sum rounds at every step, so only within tolerance).
    Raises on a mismatch."""
    import hashlib

    import torch
    import torch.distributed as dist

    from torch_mcpu_b200 import symm

    shard.front()
    part = shard.partial().clone()
    gathered = torch.empty(world * part.size(0), part.size(1), dtype=part.dtype, device="mcpu")
    dist.all_gather_into_tensor(gathered, part)
    fused = symm.mm_allreduce(shard.act, shard.wd, win).clone()
    nccl = part.clone()
    dist.all_reduce(nccl)
    torch.mcpu.synchronize()
    fused_cpu = fused.cpu()
    digest = hashlib.blake2b(fused_cpu.view(torch.int16).numpy().tobytes(), digest_size=16).hexdigest()
    digests = [None] * world
    dist.all_gather_object(digests, digest)
    result = {"ranks_identical": len(set(digests)) == 1}
    if pg is not None and dist.get_rank() == 0:
        parts = gathered.cpu().view(world, part.size(0), part.size(1))
        acc = parts[0].float()
        for r in range(1, world):
            acc = acc + parts[r].float()
        want = acc.to(torch.bfloat16)
        ndiff = int((fused_cpu.view(torch.int16) != want.view(torch.int16)).sum())
        nccl_cpu = nccl.cpu().float()
        rel = float((nccl_cpu - want.float()).norm() / want.float().norm().clamp_min(1e-30))
        result.update({"fused_vs_fp32_rank_order_sum_differing_elements": ndiff,
                       "nccl_vs_fp32_sum_rel_frobenius": rel})
    ok = torch.tensor([0 if result["ranks_identical"] and result.get(
        "fused_vs_fp32_rank_order_sum_differing_elements", 0) == 0 and result.get(
        "nccl_vs_fp32_sum_rel_frobenius", 0.0) < 1e-2 else 1], dtype=torch.int32)
    dist.all_reduce(ok, op=dist.ReduceOp.MAX)
    if int(ok.item()) != 0:
        raise SystemExit(f"bench: fused down projection + all-reduce check failed: {result}")
    result["passed"] = True
    return result


def tp_case(name, rank, world, pg, steps, warmup, peaks):
    """One TP MLP case at TP = N: the step (rms_norm if the block has one,
    gate/up GEMM + SwiGLU, down projection + SUM all-reduce) replayed from a
    CUDA graph, fused over NVLink at N > 1 with the mm + NCCL step timed
    beside it; rank 0 also times the whole block at TP=1 on its own GPU
    (the anchor of the scaling efficiency).  Whole-job TFLOP/s over the
    slowest rank's CUDA-event time."""
    import torch

    import configs as C
    from torch_mcpu_b200 import ops, symm

    cfg = getattr(C, MLP_CASES[name])
    shard = _Shard(cfg, world, rank)

    def step_nccl():
        shard.front()
        y = shard.partial()
        if pg is not None:
            pg.all_reduce(y)

    nccl_ms = _graph_ms(step_nccl, pg, steps, warmup)
    ms, mode, check = nccl_ms, "mm", None
    if world > 1:
        win = symm.SymmetricWindow(symm.window_bytes(cfg.T, cfg.H, world))

        def step_fused():
            shard.front()
            symm.mm_allreduce(shard.act, shard.wd, win)

        ms = _graph_ms(step_fused, pg, steps, warmup)
        mode = "down projection + all-reduce fused over NVLink (mm_allreduce, symmetric window)"
        torch.mcpu.synchronize()
        if ops.device_error():
            raise SystemExit("bench: mm_allreduce: a bounded wait ran out during the TP leg")
        check = _check_fused(shard, win, world, pg)
        win.close()
    del shard
    # TP=1 anchor: the whole block on rank 0's GPU alone, same job
    tp1_ms = ms
    if world > 1:
        if rank == 0:
            full = _Shard(cfg, 1, 0)

            def step_one():
                full.front()
                full.partial()

            tp1_ms = _graph_ms(step_one, None, steps, warmup)
            del full
        barrier(pg)
        t = torch.tensor([tp1_ms], dtype=torch.float64)
        pg.broadcast(t, src=0)
        tp1_ms = float(t.item())
    flops = 2 * cfg.T * cfg.H * cfg.I * 3
    whole = flops / (ms * 1e-3) / 1e12
    per_gpu = whole / world
    out = {
        "config": f"{'pre-rms_norm + ' if cfg.pre_norm else ''}SwiGLU MLP bf16 H={cfg.H} I={cfg.I} T={cfg.T} "
                  f"TP={world} (gate/up column-parallel, down row-parallel; {mode}; step replayed from a CUDA graph)",
        "ms_per_step": round(ms, 4),
        "nccl_ms_per_step": round(nccl_ms, 4),
        "tp1_ms": round(tp1_ms, 4),
        "scaling_efficiency": round(tp1_ms / (world * ms), 4),
        "tflops": round(whole, 1),
        "per_gpu_tflops": round(per_gpu, 1),
        "frac_of_bf16_peak": round(per_gpu / peaks["bf16_tflops"], 4),
        "frac_of_bf16_sustained": round(per_gpu / peaks["bf16_tflops_sustained"], 4),
        "peak_kind": peaks["kind"],
        "steps": steps,
        "flops_per_step": flops,
    }
    if cfg.T <= 256:
        # small-batch step: the weights' bytes bound it as much as the FLOPs
        wbytes = 3 * cfg.H * cfg.I * 2 // world
        out["weight_bytes_per_gpu"] = wbytes
        out["weight_gbs_per_gpu"] = round(wbytes / (ms * 1e-3) / 1e9, 1)
    if check is not None:
        out["fused_check"] = check
    return out


def tp_mlp_leg(rank, world, pg, steps, warmup, cases):
    peaks = _bf16_peaks()
    return {name: tp_case(name, rank, world, pg, steps, warmup, peaks) for name in cases}


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


def _graph_us(stream, launch, reps, per_graph):
    """us per launch of `launch(i)` replayed from a CUDA graph of per_graph
    launches (after 3 eager warm-ups and one untimed replay)."""
    import torch

    with torch.cuda.stream(stream):
        for i in range(3):
            launch(i)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(per_graph):
            launch(i)
    _upload(graph, stream)
    with torch.cuda.stream(stream):
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
    e1.synchronize()
    del graph
    return e0.elapsed_time(e1) * 1e3 / (reps * per_graph)


def moe_leg(dev, ids, stream, bufs, bias, reps=8, per_graph=32):
    """MoE dispatch after the router.  (1) moe_align_block_size alone on the
    router's own topk_ids [65536, 8] (256 experts, block 64): time per call
    and GB/s of its algorithmic bytes (ids read once, sorted ids and block
    experts written once).  (2) Router + dispatch per batch over the
    router's rotating inputs: the router alone, the router then
    moe_align_block_size (three launches), and mcpu_grouped_topk_moe_align
    (one launch), whose outputs are first checked equal to the two calls'."""
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

    def align(i, src=ids):
        _lib.check(lib.mcpu_moe_align_block_size(src.data_ptr(), numel, E_, bs, srt.data_ptr(), cap, eid.data_ptr(),
                                                 nblk, npad.data_ptr(), work.data_ptr(), wsb.value,
                                                 stream.cuda_stream), "moe_align_block_size")

    us = _graph_us(stream, align, reps, per_graph)
    nbytes = numel * 4 + cap * 4 + nblk * 4 + 4
    gbs = nbytes / (us * 1e-6) / 1e9
    out = {"shape": f"topk_ids int32 [{numel // 8}, 8] from the router, {E_} experts, block {bs}",
           "us_per_call": round(us, 2), "launches_per_call": 2, "algorithmic_bytes": nbytes,
           "achieved_gbs": round(gbs, 1), "peak_gbs": peak, "frac": round(gbs / peak, 4), "peak_kind": peak_kind}

    # router + dispatch over the rotating inputs
    w2 = torch.empty(T, K, dtype=torch.float32, device=dev)
    ids2 = torch.empty(T, K, dtype=torch.int32, device=dev)
    fwsb = ctypes.c_uint64()
    _lib.check(lib.mcpu_grouped_topk_moe_align_workspace_bytes(T, E_, K, ctypes.byref(fwsb)), "fused workspace")
    fwork = torch.zeros(fwsb.value, dtype=torch.uint8, device=dev)
    fsrt = torch.empty(cap, dtype=torch.int32, device=dev)
    feid = torch.empty(nblk, dtype=torch.int32, device=dev)
    fnpad = torch.empty(1, dtype=torch.int32, device=dev)

    def route(i):
        _lib.check(lib.mcpu_grouped_topk(bufs[i % N_BUFFERS].data_ptr(), 0, T, E_, G, TG, K, 1, 2.5,
                                         bias.data_ptr(), 1, w2.data_ptr(), ids2.data_ptr(), stream.cuda_stream),
                   "grouped_topk")

    def route_then_align(i):
        route(i)
        align(i, ids2)

    def fused(i):
        _lib.check(lib.mcpu_grouped_topk_moe_align(
            bufs[i % N_BUFFERS].data_ptr(), 0, T, E_, G, TG, K, 1, 2.5, bias.data_ptr(), 1, w2.data_ptr(),
            ids2.data_ptr(), bs, fsrt.data_ptr(), cap, feid.data_ptr(), nblk, fnpad.data_ptr(), fwork.data_ptr(),
            fwsb.value, stream.cuda_stream), "grouped_topk_moe_align")

    with torch.cuda.stream(stream):
        route_then_align(1)
        fused(1)
    stream.synchronize()
    if not (torch.equal(fsrt, srt) and torch.equal(feid, eid) and torch.equal(fnpad, npad)):
        raise SystemExit("bench: fused router + dispatch differs from the router then moe_align_block_size")
    us_router = _graph_us(stream, route, reps, per_graph)
    us_two = _graph_us(stream, route_then_align, reps, per_graph)
    us_fused = _graph_us(stream, fused, reps, per_graph)
    out["router_then_dispatch"] = {
        "config": f"T={T} E={E_} topk={K} block {bs}, {N_BUFFERS} rotating {T * E_ * 4 / 1e6:.1f} MB inputs, "
                  f"graph replay of {per_graph} calls",
        "router_us": round(us_router, 2),
        "router_then_moe_align_us": round(us_two, 2),
        "fused_us": round(us_fused, 2),
        "fused_minus_router_us": round(us_fused - us_router, 2),
        "launches": {"router": 1, "router_then_moe_align": 3, "fused": 1},
        "fused_mtok_s": round(T / (us_fused * 1e-6) / 1e6, 1),
    }
    return out


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
def _upload(graph, stream):
    """Uploads an instantiated CUDA graph to the device (cuGraphUpload), so
    that its first replay inside a timed region carries no upload cost."""
    cu = ctypes.CDLL("libcuda.so.1")
    cu.cuGraphUpload.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    cu.cuGraphUpload.restype = ctypes.c_int
    rc = cu.cuGraphUpload(ctypes.c_void_p(int(graph.raw_cuda_graph_exec())), ctypes.c_void_p(stream.cuda_stream))
    if rc != 0:
        raise SystemExit(f"bench: cuGraphUpload failed ({rc})")


def _replay_plan(n, per_graph=GRAPH_STEPS):
    """Exactly n launches as full graphs of per_graph launches plus one
    remainder graph: (full replays, remainder size)."""
    g = min(per_graph, n)
    return g, n // g, n % g


def router_sweep_leg(lib, dev, stream, reps=20):
    """Latency per call at small batches (graph replay of 64 launches, inputs
    resident) for the DeepSeek-V3 router at T in {1, 16, 256, 4096}, and the
    softmax variant (160 experts, 8 groups, top-3 groups, top-6, no bias) at
    65536 tokens over rotating inputs larger than L2, with its roofline at
    160 x 4 + 6 x 8 = 688 algorithmic bytes per token."""
    import torch

    import configs as C

    peak, peak_kind = measured_peaks()
    out = {"latency_us": {}}

    def timed(launch, n_in, per_graph=64):
        with torch.cuda.stream(stream):
            for i in range(3):
                launch(i)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(per_graph):
                launch(i)
        with torch.cuda.stream(stream):
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        del graph
        return e0.elapsed_time(e1) * 1e3 / (reps * per_graph)

    for t in (1, 16, 256, 4096):
        cfg = C.deepseek_v3(t)
        gating, bias = C.router_inputs(cfg)
        g, b = gating.to(dev), bias.to(dev)
        w = torch.empty(t, K, dtype=torch.float32, device=dev)
        ids = torch.empty(t, K, dtype=torch.int32, device=dev)

        def launch(i, g=g, b=b, w=w, ids=ids, t=t):
            rc = lib.mcpu_grouped_topk(g.data_ptr(), 0, t, E, G, TG, K, 1, 2.5, b.data_ptr(), 1, w.data_ptr(),
                                       ids.data_ptr(), stream.cuda_stream)
            if rc != 0:
                from torch_mcpu_b200 import _lib

                _lib.check(rc, "grouped_topk")

        out["latency_us"][f"T{t}"] = round(timed(launch, 1), 2)
    out["latency_config"] = "sigmoid+bias E=256 G=8 topk_group=4 topk=8, us per call, graph replay of 64 calls"

    # softmax variant, throughput at 65536 tokens
    cfg = C.softmax160(T)
    E2, K2 = cfg.E, cfg.K
    gating, _ = C.router_inputs(cfg)
    bufs = [gating.to(dev)]
    for i in range(1, N_BUFFERS):
        gg = torch.Generator(device=dev).manual_seed(200 + i)
        bufs.append(torch.randn(T, E2, generator=gg, device=dev))
    w = torch.empty(T, K2, dtype=torch.float32, device=dev)
    ids = torch.empty(T, K2, dtype=torch.int32, device=dev)

    def launch_sm(i):
        rc = lib.mcpu_grouped_topk(bufs[i % N_BUFFERS].data_ptr(), 0, T, E2, cfg.G, cfg.TG, K2, 0, 1.0, None, 0,
                                   w.data_ptr(), ids.data_ptr(), stream.cuda_stream)
        if rc != 0:
            from torch_mcpu_b200 import _lib

            _lib.check(rc, "grouped_topk")

    us = timed(launch_sm, N_BUFFERS)
    nbytes = T * (E2 * 4 + K2 * 8)
    gbs = nbytes / (us * 1e-6) / 1e9
    out["softmax160"] = {
        "config": f"softmax E={E2} G={cfg.G} topk_group={cfg.TG} topk={K2}, no bias, T={T}, "
                  f"{N_BUFFERS} rotating {T * E2 * 4 / 1e6:.1f} MB inputs",
        "us_per_call": round(us, 2),
        "mtok_s": round(T / (us * 1e-6) / 1e6, 1),
        "algorithmic_bytes": nbytes,
        "achieved_gbs": round(gbs, 1),
        "peak_gbs": peak,
        "frac": round(gbs / peak, 4),
        "peak_kind": peak_kind,
    }
    return out


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

    # exactly K timed launches: full graphs of up to GRAPH_STEPS launches plus
    # a remainder graph, rotating over the input buffers
    per, full, rem = _replay_plan(a.steps)
    graph = torch.cuda.CUDAGraph()
    graph_rem = torch.cuda.CUDAGraph() if rem else None
    with torch.cuda.stream(stream):
        for i in range(3):
            launch(i)
    stream.synchronize()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(per):
            launch(i)
    if graph_rem is not None:
        with torch.cuda.graph(graph_rem, stream=stream):
            for i in range(rem):
                launch(per + i)
    _upload(graph, stream)
    if graph_rem is not None:
        _upload(graph_rem, stream)
    stream.synchronize()
    steps = full * per + rem

    exact_before = ctypes.c_ulonglong(0)
    lib.mcpu_grouped_topk_exact_rows(ctypes.byref(exact_before), 1)
    busy = []  # (start, end) of every timed region, for the clock record
    clk = ClockSampler(local).__enter__()
    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            launch(i)
    stream.synchronize()
    barrier(pg)
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.monotonic()
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(full):
            graph.replay()
        if graph_rem is not None:
            graph_rem.replay()
        ev1.record(stream)
    ev1.synchronize()
    torch.cuda.synchronize(dev)
    busy.append((t0, time.monotonic()))
    barrier(pg)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(pg, ms)
    exact = ctypes.c_ulonglong(0)
    lib.mcpu_grouped_topk_exact_rows(ctypes.byref(exact), 0)
    exact_per_step = exact.value / (steps + a.warmup)
    del graph, graph_rem

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
    e2e_steps = max(3, min(a.steps, 200))
    if "e2e" in a.legs:
        for i in range(4):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        barrier(pg)
        t0 = time.monotonic()
        ev0.record(s_in)
        for i in range(e2e_steps):
            e2e_step(i)
        ev1.record(s_out)
        ev1.synchronize()
        torch.cuda.synchronize(dev)
        busy.append((t0, time.monotonic()))
        barrier(pg)
        e2e_ms = max_over_ranks(pg, ev0.elapsed_time(ev1)) / e2e_steps

    def leg(name, fn):
        t0 = time.monotonic()
        r = fn()
        busy.append((t0, time.monotonic()))
        return r

    sweep = leg("sweep", lambda: router_sweep_leg(lib, dev, stream)) if "sweep" in a.legs else None
    bw = leg("bw", lambda: bandwidth_leg(dev)) if "bw" in a.legs else None
    moe = leg("moe", lambda: moe_leg(dev, ids, stream, bufs, bias)) if "moe" in a.legs else None
    sampler = leg("sampler", lambda: sampler_leg(dev)) if "sampler" in a.legs else None
    mlp = None
    if "mlp" in a.legs:
        cases = [c for c in a.mlp_cases.split(",") if c]
        mlp = leg("mlp", lambda: tp_mlp_leg(rank, world, pg, steps=max(10, min(a.steps, 50)), warmup=3,
                                            cases=cases))
    clk.__exit__(None, None, None)

    if rank == 0:
        per_step = ms_max / steps
        peak, peak_kind = measured_peaks()
        achieved = BYTES_PER_TOKEN * T / (per_step * 1e-3) / 1e9
        traffic = profiled_traffic("grouped_topk_T65536_E256.md")
        clocks = clk.summary(busy, "the timed regions of every leg (router, e2e, sweep, bandwidth, "
                                   "dispatch, sampler and MLP legs)")
        clocks["router_timed_region"] = clk.summary(busy[:1], "the router's timed region")
        line = {
            "metric": METRIC,
            "value": round(T * world / (per_step * 1e-3) / 1e6, 2),
            "unit": "Mtok/s",
            "n_gpus": world,
            "steps": steps,
            "warmup": a.warmup,
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
                "steps": e2e_steps,
                "path": "per step: orMemcpyAsync H2D (pinned) -> mcpu_grouped_topk -> orMemcpyAsync D2H (pinned); "
                        "two buffer sets on copy-in / router / copy-out streams, so step i+1's input copy "
                        "overlaps step i's router",
            },
            "clocks": clocks,
            "gpu_launches": steps,
            "exact_path_rows_per_step": round(exact_per_step, 2),
            "router_sweep": sweep,
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
    """The reference arm: the reference's router op chain on the host cores
    (rank 0 only), K timed steps of the full batch after W warm-ups, with
    the path's other legs timed within --cpu-seconds each."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    legs = cpu_legs(a.cpu_seconds, steps=a.steps, warmup=a.warmup)
    r = legs["router"]
    host = legs["host"]
    base = {"value": r["value"], "unit": "Mtok/s", "cores": host["torch_threads"], "kind": "port",
            "sample": r["sample"] + f"; host: {host['nproc']} x {host['cpu_model']}"}
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": r["value"],
        "unit": "Mtok/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": r["ms_per_batch"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) logits, N(0,0.01) bias)",
        "config": workload_config(1),
        "cpu_baseline": base,
        "e2e": {"value": r["value"], "unit": "Mtok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_legs": legs,
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
