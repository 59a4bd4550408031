"""Host logic of the tensor-parallel MLP on CPU with two gloo ranks.

Each rank evaluates its shard with the oracle and the partial outputs are
summed by a gloo all-reduce (example/01_mlp_tp4/run.py:106-126 structure):
the result must equal the unsharded computation, and every rank must hold
the same output (run.py:315-344).  No GPU involved.
"""

import os
import tempfile

import numpy as np
import torch


def _rank(rank, world, init_file, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "tests", "golden")]
    import torch.distributed as dist

    import configs as C
    import oracle

    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    cfg = C.MLP_TINY_NORM
    x, rms_w, wgu, wd = C.mlp_weights(cfg, world, rank)
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    h = oracle.rms_norm_bf16(bits(x), bits(rms_w), C.RMS_EPS)
    a = oracle.silu_and_mul_bf16(oracle.gemm_bf16(h, bits(wgu)))
    y = torch.from_numpy(oracle.bf16_bits_to_f32(oracle.gemm_bf16(a, bits(wd))).copy())
    dist.all_reduce(y)
    q.put((rank, y.numpy()))
    dist.destroy_process_group()


def test_two_rank_tp_step_equals_unsharded():
    import torch.multiprocessing as mp

    import configs as C
    import oracle

    fd, init_file = tempfile.mkstemp(prefix="mcpu_tp_")
    os.close(fd)
    os.unlink(init_file)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, init_file, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_array_equal(out[0], out[1])
    x, rms_w, wgu1, wd1 = C.mlp_weights(C.MLP_TINY_NORM, 1, 0)
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    full = oracle.bf16_bits_to_f32(oracle.tp_mlp_bf16(bits(x), [bits(wgu1)], [bits(wd1)], bits(rms_w), C.RMS_EPS))
    assert np.linalg.norm(out[0] - full) / np.linalg.norm(full) < 1e-2
