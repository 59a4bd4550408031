"""The "mcpu" ProcessGroup over NCCL, on two or more GPUs of one box.

Known answers as in the reference's tests/test_distributed.py (all_reduce of
rank + 1 over 2 ranks = 3.0, test_distributed.py:300) plus one
tensor-parallel SwiGLU MLP step against the oracle.  Ranks are spawned
processes; the group uses "cpu:gloo,mcpu:mcpu" like the reference.
"""

import os
import tempfile

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, init_file, q):
    try:
        import sys

        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "tests", "golden")]
        import datetime

        import torch.distributed as dist

        import torch_mcpu_b200.device  # noqa: F401

        torch.mcpu.set_device(rank)
        dist.init_process_group("cpu:gloo,mcpu:mcpu", init_method=f"file://{init_file}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        t = torch.full((4,), float(rank + 1)).to("mcpu")
        dist.all_reduce(t)
        torch.mcpu.synchronize()
        r1 = t.cpu().tolist()
        b = torch.full((3,), float(rank)).to("mcpu")
        dist.broadcast(b, src=1)
        torch.mcpu.synchronize()
        r2 = b.cpu().tolist()
        inp = torch.full((2,), float(rank)).to("mcpu")
        out = torch.empty(2 * world, device="mcpu")
        dist.all_gather_into_tensor(out, inp)
        torch.mcpu.synchronize()
        r3 = out.cpu().tolist()
        dist.barrier()
        # one TP step of the gated MLP (tiny config), partials summed by NCCL
        import configs as C
        from torch_mcpu_b200 import ops

        cfg = C.MLP_TINY
        x, _, wgu, wd = C.mlp_weights(cfg, world, rank)
        xm, wgum, wdm = x.to("mcpu"), wgu.to("mcpu"), wd.to("mcpu")
        act = torch.ops.mcpu.gemm_swiglu(xm, wgum.view(2, -1, 128, wgu.shape[1]).transpose(0, 1)
                                          .reshape(wgu.shape).contiguous())
        y = torch.mm(act, wdm.t())
        dist.all_reduce(y)
        torch.mcpu.synchronize()
        # the same down projection + all-reduce fused over a symmetric
        # window, twice in a row (the kernel resets its counters), then a
        # TP=8-sized shard [2048 x 1792] x [4096 x 1792]^T against NCCL
        from torch_mcpu_b200 import symm

        win = symm.SymmetricWindow(symm.window_bytes(2048, 4096, world))
        f1 = symm.mm_allreduce(act, wdm, win).cpu()
        f2 = symm.mm_allreduce(act, wdm, win).cpu()
        g = torch.Generator().manual_seed(100 + rank)
        a = torch.randn(2048, 1792, generator=g).to(torch.bfloat16).to("mcpu")
        b = (0.02 * torch.randn(4096, 1792, generator=g)).to(torch.bfloat16).to("mcpu")
        big = symm.mm_allreduce(a, b, win).cpu()
        big_nccl = torch.mm(a, b.t())
        dist.all_reduce(big_nccl)
        big_nccl = big_nccl.cpu()
        torch.mcpu.synchronize()
        err = ops.device_error()
        win.close()
        fused = (f1.view(torch.int16).numpy(), f2.view(torch.int16).numpy(), big.view(torch.int16).numpy(),
                 big_nccl.view(torch.int16).numpy(), err)
        q.put((rank, r1, r2, r3, y.cpu().view(torch.int16).numpy(), fused))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, "error", traceback.format_exc(), None, None, None))


def test_process_group_collectives_and_tp_step():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import configs as C
    import oracle

    world = 2
    fd, init_file = tempfile.mkstemp(prefix="mcpu_pg_")
    os.close(fd)
    os.unlink(init_file)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, init_file, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, *rest = q.get(timeout=300)
        res[rank] = rest
    for p in procs:
        p.join(timeout=120)
    for rank, (r1, r2, r3, y, _) in res.items():
        assert r1 != "error", r2
        assert r1 == [3.0] * 4
        assert r2 == [1.0] * 3
        assert r3 == [0.0, 0.0, 1.0, 1.0]
    shards = [C.mlp_weights(C.MLP_TINY, world, r) for r in range(world)]
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    ref = oracle.bf16_bits_to_f32(oracle.tp_mlp_bf16(bits(shards[0][0]), [bits(s[2]) for s in shards],
                                                     [bits(s[3]) for s in shards], None, exp_mode=oracle.EXP_CR))
    for rank in range(world):
        got = oracle.bf16_bits_to_f32(res[rank][3].view(np.uint16))
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-2
    np.testing.assert_array_equal(res[0][3], res[1][3])
    # fused down projection + all-reduce: the same bits on every rank, on
    # repeated calls, and within bf16 rounding of NCCL's sum
    f = [res[r][4] for r in range(world)]
    for r in range(world):
        assert f[r][4] == 0, "device error flag set"
        np.testing.assert_array_equal(f[r][0], f[0][0])
        np.testing.assert_array_equal(f[r][1], f[0][0])
        np.testing.assert_array_equal(f[r][2], f[0][2])
    got = oracle.bf16_bits_to_f32(f[0][0].view(np.uint16))
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-2
    big = oracle.bf16_bits_to_f32(f[0][2].view(np.uint16)).astype(np.float64)
    nccl = oracle.bf16_bits_to_f32(f[0][3].view(np.uint16)).astype(np.float64)
    # two bf16 roundings apart at most (NCCL may round after each hop)
    assert np.all(np.abs(big - nccl) <= 2 ** -7 * np.maximum(np.abs(nccl), np.abs(big)) + 1e-6)
