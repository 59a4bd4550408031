"""Router + expert dispatch in one call (mcpu_grouped_topk_moe_align) on the
GPU.  Its router outputs must equal mcpu_grouped_topk's bit for bit, and its
dispatch outputs (sorted_token_ids, expert_ids, num_tokens_post_pad) the
oracle's counting sort of those ids: integer work, identical outputs.

Covers the one-launch path (DeepSeek-V3's router shape) at the benchmark
size and at ragged sizes (1 token, partial tiles, more tiles than one pass
of the grid), a large batch whose CTAs hold more ids than their staging
buffer (placed straight from registers), skewed routing (every token on the
same 8 experts), near-tie rows that take the router's exact paths, repeated
calls on one workspace, the two-launch path (softmax router, and the fused
shape with the fusion switched off), and the bounded grid barrier: a
workspace whose arrival counts are wrong makes every CTA's wait run out,
which must be reported through mcpu_device_error and leave the context
usable."""

import ctypes
import os

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu


def _lib():
    from torch_mcpu_b200 import _lib

    return _lib


def _ws_bytes(T, E, K):
    L = _lib()
    nb = ctypes.c_uint64()
    L.check(L.load().mcpu_grouped_topk_moe_align_workspace_bytes(T, E, K, ctypes.byref(nb)), "workspace bytes")
    return nb.value


def _fused(cfg, g, bias, bs, ws=None):
    """One mcpu_grouped_topk_moe_align call through the C-ABI; returns the
    five outputs (device tensors)."""
    L = _lib()
    lib = L.load()
    T, E = g.shape
    numel = T * cfg.K
    cap = min(numel + E * (bs - 1), numel * bs)
    nblocks = -(-cap // bs)
    dev = g.device
    w = torch.empty(T, cfg.K, dtype=torch.float32, device=dev)
    ids = torch.empty(T, cfg.K, dtype=torch.int32, device=dev)
    s = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    e = torch.empty(max(nblocks, 1), dtype=torch.int32, device=dev)
    n = torch.empty(1, dtype=torch.int32, device=dev)
    need = _ws_bytes(T, E, cfg.K)
    if ws is None:
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    assert ws.numel() >= need
    rc = lib.mcpu_grouped_topk_moe_align(
        g.data_ptr(), 0 if g.dtype == torch.float32 else 1, T, E, cfg.G, cfg.TG, cfg.K, int(cfg.renorm),
        float(cfg.scale), None if bias is None else bias.data_ptr(), 1 if cfg.scoring == "sigmoid" else 0,
        w.data_ptr(), ids.data_ptr(), bs, s.data_ptr(), cap, e.data_ptr(), nblocks, n.data_ptr(),
        ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    L.check(rc, "grouped_topk_moe_align")
    return w, ids, s[:cap], e[:nblocks], n


def _router(cfg, g, bias):
    from torch_mcpu_b200 import ops

    return ops.grouped_topk(g, g, cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring, cfg.scale, bias)


def _check(cfg, g, bias, bs, got):
    w, ids, s, e, n = got
    rw, rids = _router(cfg, g, bias)
    torch.cuda.synchronize()
    assert torch.equal(ids, rids)
    assert torch.equal(w.view(torch.int32), rw.view(torch.int32))  # bit for bit
    ws_, we_, wn_ = oracle.moe_align_block_size(ids.cpu().numpy(), g.shape[1], bs, sorted_capacity=s.numel())
    assert int(n.cpu()[0]) == wn_
    np.testing.assert_array_equal(s.cpu().numpy(), ws_)
    np.testing.assert_array_equal(e.cpu().numpy(), we_[: e.numel()])


def _inputs(cfg):
    gating, bias = C.router_inputs(cfg)
    return gating.cuda(), None if bias is None else bias.cuda()


@pytest.mark.parametrize("bs", [16, 64, 128])
def test_fused_deepseek_v3_benchmark_size(bs):
    from torch_mcpu_b200 import ops

    ops.device_error(reset=True)
    cfg = C.deepseek_v3(65536)
    g, b = _inputs(cfg)
    _check(cfg, g, b, bs, _fused(cfg, g, b, bs))
    assert ops.device_error() == 0


@pytest.mark.parametrize("T", [1, 7, 9, 223, 4095, 8193, 100003])
def test_fused_ragged_sizes(T):
    cfg = C.deepseek_v3(T, seed=T)
    g, b = _inputs(cfg)
    _check(cfg, g, b, 64, _fused(cfg, g, b, 64))


def test_fused_large_batch_many_tiles_per_cta():
    """1,000,000 tokens: about 845 tiles (54,000 ids) per CTA, more than the
    staging buffer holds and close to the 16-bit per-CTA count."""
    cfg = C.deepseek_v3(1_000_000, seed=3)
    g, b = _inputs(cfg)
    _check(cfg, g, b, 64, _fused(cfg, g, b, 64))


def test_fused_skewed_every_token_on_the_same_experts():
    """A bias that sends every token to experts 0..7: eight runs of T ids,
    all other experts empty."""
    T = 200_000
    cfg = C.deepseek_v3(T, seed=11)
    g, b = _inputs(cfg)
    b = b.clone()
    b[:8] += 100.0
    got = _fused(cfg, g, b, 64)
    _check(cfg, g, b, 64, got)
    assert int(got[4].cpu()[0]) == 8 * (-(-T // 64) * 64)


def test_fused_near_ties_take_the_exact_paths():
    cfg = C.RouterCfg("ties_many", 4000, 256, 8, 4, 8, "sigmoid", True, True, 2.5)
    gen = torch.Generator().manual_seed(4)
    gating = torch.randn(4000, 256, generator=gen)
    gating[0::3] = 0.0
    gating[1::3, 64:96] = 3.0
    gating[2::3, :] = torch.randn(1, 256, generator=gen).round()
    g, b = gating.cuda(), torch.zeros(256, device="cuda")
    _check(cfg, g, b, 16, _fused(cfg, g, b, 16))


def test_fused_repeated_calls_on_one_workspace():
    from torch_mcpu_b200 import ops

    ops.device_error(reset=True)
    ws = torch.zeros(_ws_bytes(30000, 256, 8), dtype=torch.uint8, device="cuda")
    for seed in range(4):
        cfg = C.deepseek_v3(30000 - 1000 * seed, seed=seed)
        g, b = _inputs(cfg)
        _check(cfg, g, b, 32, _fused(cfg, g, b, 32, ws))
    head = ws[:12].view(torch.int32).cpu().tolist()
    assert head[0] == 4  # one generation per call
    assert min(head[1], head[2]) == 0  # the next call's arrival count is clear
    assert ops.device_error() == 0


def test_two_launch_paths_agree():
    """The softmax router (no fused path) and the fused shape with the
    fusion switched off run the router, then the dispatch's two launches."""
    cfg = C.softmax160(5000, True)
    g, b = _inputs(cfg)
    _check(cfg, g, b, 64, _fused(cfg, g, b, 64))
    cfg = C.deepseek_v3(20000, seed=9)
    g, b = _inputs(cfg)
    fused = _fused(cfg, g, b, 64)
    os.environ["MCPU_DISPATCH_UNFUSED"] = "1"
    try:
        two = _fused(cfg, g, b, 64)
    finally:
        del os.environ["MCPU_DISPATCH_UNFUSED"]
    for a, c in zip(fused, two):
        assert torch.equal(a.view(torch.int32), c.view(torch.int32))
    _check(cfg, g, b, 64, two)


def test_python_wrapper_matches_the_two_ops():
    from torch_mcpu_b200 import ops

    cfg = C.deepseek_v3(12345, seed=5)
    g, b = _inputs(cfg)
    w, ids, s, e, n = ops.grouped_topk_moe_align(g, g, 8, True, 8, 4, "sigmoid", 2.5, b, block_size=64)
    rw, rids = ops.grouped_topk(g, g, 8, True, 8, 4, "sigmoid", 2.5, b)
    rs, re_, rn = ops.moe_align_block_size(rids, 64, 256)
    assert torch.equal(ids, rids) and torch.equal(w, rw)
    assert torch.equal(s, rs) and torch.equal(e, re_) and torch.equal(n, rn)


def test_barrier_wait_runs_out_and_is_reported():
    """Arrival counts of 1000 in the workspace: the count never equals the
    number of CTAs, so every CTA's wait gives up after its time bound and
    the call reports it; with the workspace zeroed again the next call is
    correct."""
    from torch_mcpu_b200 import ops

    cfg = C.deepseek_v3(4096, seed=2)
    g, b = _inputs(cfg)
    ws = torch.zeros(_ws_bytes(4096, 256, 8), dtype=torch.uint8, device="cuda")
    ws[4:12].view(torch.int32).fill_(1000)  # both parities' arrival counts
    ops.device_error(reset=True)
    _fused(cfg, g, b, 64, ws)
    torch.cuda.synchronize()
    assert ops.device_error(reset=True) != 0
    ws.zero_()
    _check(cfg, g, b, 64, _fused(cfg, g, b, 64, ws))
    assert ops.device_error() == 0


def test_rejects_bad_arguments():
    cfg = C.deepseek_v3(64)
    g, b = _inputs(cfg)
    L = _lib()
    lib = L.load()
    ws = torch.zeros(_ws_bytes(64, 256, 8), dtype=torch.uint8, device="cuda")
    w = torch.empty(64, 8, device="cuda")
    ids = torch.empty(64, 8, dtype=torch.int32, device="cuda")
    n = torch.empty(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    small = torch.empty(16, dtype=torch.int32, device="cuda")
    rc = lib.mcpu_grouped_topk_moe_align(g.data_ptr(), 0, 64, 256, 8, 4, 8, 1, 2.5, b.data_ptr(), 1, w.data_ptr(),
                                         ids.data_ptr(), 64, small.data_ptr(), 16, small.data_ptr(), 16,
                                         n.data_ptr(), ws.data_ptr(), ws.numel(), st)
    assert rc != 0 and b"sorted_token_ids holds" in lib.mcpuGetLastErrorString()
    cap = min(64 * 8 + 256 * 63, 64 * 8 * 64)
    s = torch.empty(cap, dtype=torch.int32, device="cuda")
    e = torch.empty(-(-cap // 64), dtype=torch.int32, device="cuda")
    rc = lib.mcpu_grouped_topk_moe_align(g.data_ptr(), 0, 64, 256, 8, 4, 8, 1, 2.5, b.data_ptr(), 1, w.data_ptr(),
                                         ids.data_ptr(), 64, s.data_ptr(), cap, e.data_ptr(), e.numel(),
                                         n.data_ptr(), ws.data_ptr(), 8, st)
    assert rc != 0 and b"workspace of" in lib.mcpuGetLastErrorString()
