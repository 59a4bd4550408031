"""MoE dispatch (mcpu_moe_align_block_size) on the GPU against the oracle:
the router's own topk_ids at the DeepSeek-V3 shape (65536 tokens, top-8 of
256 experts), the softmax router's (160 experts, top-6), skewed and tiny
inputs, no padding (block 1), more experts than entries, out-of-range
entries, and the mcpu custom op with vLLM's schema.  Integer work: the
outputs must be identical."""

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu


def _check(ids_np, E, bs, got):
    s, e, n = (t.cpu().numpy() for t in got)
    ws, we, wn = oracle.moe_align_block_size(ids_np, E, bs, sorted_capacity=len(s))
    assert int(n[0]) == wn
    np.testing.assert_array_equal(s, ws)
    np.testing.assert_array_equal(e, we[: len(e)])


def _router_ids(cfg):
    from torch_mcpu_b200 import ops

    gating, bias = C.router_inputs(cfg)
    g = gating.cuda()
    _, ids = ops.grouped_topk(g, g, cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring, cfg.scale,
                              None if bias is None else bias.cuda())
    return ids


@pytest.mark.parametrize("bs", [16, 64, 128])
def test_router_ids_deepseek_v3(bs):
    from torch_mcpu_b200 import ops

    ops.device_error(reset=True)
    ids = _router_ids(C.deepseek_v3(65536))
    got = ops.moe_align_block_size(ids, bs, 256)
    _check(ids.cpu().numpy(), 256, bs, got)
    assert ops.device_error() == 0


def test_router_ids_softmax160():
    from torch_mcpu_b200 import ops

    ids = _router_ids(C.softmax160(4096, True))
    got = ops.moe_align_block_size(ids, 64, 160, pad_sorted_ids=True)
    _check(ids.cpu().numpy(), 160, 64, got)


@pytest.mark.parametrize("T,K,E,bs,kind", [(1, 8, 256, 16, "rand"), (3, 4, 1024, 32, "rand"),
                                           (5000, 8, 256, 64, "skew"), (4097, 2, 8, 1, "rand"),
                                           (12345, 8, 64, 256, "rand"), (2, 2, 1, 4, "rand")])
def test_shapes_and_distributions(T, K, E, bs, kind):
    from torch_mcpu_b200 import ops

    g = np.random.default_rng(T + E)
    if kind == "skew":
        ids = np.where(g.random((T, K)) < 0.9, 3, g.integers(0, E, (T, K)))
    else:
        ids = g.integers(0, E, (T, K))
    t = torch.from_numpy(ids.astype(np.int32)).cuda()
    _check(ids, E, bs, ops.moe_align_block_size(t, bs, E))


def test_out_of_range_entries_flagged_and_left_out():
    from torch_mcpu_b200 import ops

    ops.device_error(reset=True)
    ids = np.array([[0, 5, -1], [1, 1, 9]], dtype=np.int32)
    got = ops.moe_align_block_size(torch.from_numpy(ids).cuda(), 2, 4)
    _check(ids, 4, 2, got)
    torch.cuda.synchronize()
    assert ops.device_error(reset=True) != 0


def test_mcpu_custom_op_schema():
    import torch_mcpu_b200.device  # noqa: F401

    g = np.random.default_rng(5)
    ids = g.integers(0, 256, (777, 8)).astype(np.int32)
    numel, E, bs = ids.size, 256, 64
    cap = min(numel + E * (bs - 1), numel * bs)
    s = torch.empty(cap, dtype=torch.int32, device="mcpu")
    e = torch.empty(-(-cap // bs), dtype=torch.int32, device="mcpu")
    n = torch.empty(1, dtype=torch.int32, device="mcpu")
    torch.ops.mcpu.moe_align_block_size(torch.from_numpy(ids).to("mcpu"), E, bs, s, e, n)
    _check(ids, E, bs, (s, e, n))
    with pytest.raises(RuntimeError, match="sorted_token_ids holds"):
        torch.ops.mcpu.moe_align_block_size(torch.from_numpy(ids).to("mcpu"), E, bs, s[:10], e, n)
