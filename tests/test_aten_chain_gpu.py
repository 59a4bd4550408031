"""The generic aten registrations of the mcpu device, exercised the way the
reference's users run its hot path op by op: the grouped_topk router chain of
tests/test_grouped_topk_compile.py:15-66 (kzwrime/torch_mcpu), restated here
step by step, and vLLM's native silu_and_mul / rms_norm formulas, each on mcpu
tensors; results against the oracle (bit-exact where the chain is), and the
individual ops against torch on the CPU."""

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mcpu():
    import torch_mcpu_b200.device as d

    assert torch.mcpu.is_available()
    return d


def router_chain(gating, topk, renormalize, num_expert_group, topk_group, scoring, scale, bias):
    """The reference router's aten steps (softmax or sigmoid, bias add, group
    top-2 sum or max, group top-k, group mask by scatter, masked fill, expert
    top-k, gather, renormalise, scale) on whatever device the inputs are."""
    scores = torch.softmax(gating, dim=-1) if scoring == "softmax" else gating.sigmoid()
    T = scores.size(0)
    if bias is not None:
        unbiased = scores
        scores = scores + bias.unsqueeze(0)
        gs = scores.view(T, num_expert_group, -1).topk(2, dim=-1)[0].sum(dim=-1)
    else:
        gs = scores.view(T, num_expert_group, -1).max(dim=-1).values
    gidx = torch.topk(gs, k=topk_group, dim=-1, sorted=False)[1]
    gmask = torch.zeros_like(gs)
    gmask.scatter_(1, gidx, 1)
    smask = gmask.unsqueeze(-1).expand(T, num_expert_group, scores.size(-1) // num_expert_group).reshape(T, -1)
    masked = scores.masked_fill(~smask.bool(), float("-inf"))
    if bias is not None:
        ids = torch.topk(masked, k=topk, dim=-1, sorted=False)[1]
        w = unbiased.gather(1, ids)
    else:
        w, ids = torch.topk(masked, k=topk, dim=-1, sorted=False)
    if renormalize:
        w = w / w.sum(dim=-1, keepdim=True)
    if scale != 1.0:
        w = w * scale
    return w.to(torch.float32), ids.to(torch.int32)


def _check_router(cfg, w, ids, rtol):
    gating, bias = C.router_inputs(cfg)
    ow, oids, oties, gaps = oracle.grouped_topk(gating.numpy(), cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring,
                                                cfg.scale, None if bias is None else bias.numpy(),
                                                exp_mode=oracle.EXP_CR)
    got = np.sort(ids, 1)
    want = np.sort(oids, 1)
    bad = np.nonzero((got != want).any(1))[0]
    # a row may differ only where the oracle's own selection is an exact tie
    assert all(oties[r] for r in bad), f"{len(bad)} rows differ: {bad[:8]}"
    ok = np.setdiff1d(np.arange(cfg.T), bad)
    og = np.argsort(ids[ok], 1)
    oo = np.argsort(oids[ok], 1)
    a = np.take_along_axis(w[ok], og, 1)
    b = np.take_along_axis(ow[ok], oo, 1)
    np.testing.assert_allclose(a, b, rtol=rtol, atol=0)


def test_reference_router_chain_on_mcpu_sigmoid_bias(mcpu):
    cfg = C.deepseek_v3(1024)
    gating, bias = C.router_inputs(cfg)
    w, ids = router_chain(gating.to("mcpu"), cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring, cfg.scale,
                          bias.to("mcpu"))
    assert w.device.type == "mcpu" and ids.device.type == "mcpu"
    _check_router(cfg, w.cpu().numpy(), ids.cpu().numpy(), 1e-5)
    # the same inputs through the fused op
    fw, fids = torch.ops.mcpu.grouped_topk(gating.to("mcpu"), cfg.G, cfg.TG, cfg.K, cfg.renorm, cfg.scale,
                                           bias.to("mcpu"), "sigmoid")
    np.testing.assert_array_equal(np.sort(fids.cpu().numpy(), 1), np.sort(ids.cpu().numpy(), 1))


def test_reference_router_chain_on_mcpu_softmax(mcpu):
    cfg = C.softmax160(512, True)
    gating, _ = C.router_inputs(cfg)
    w, ids = router_chain(gating.to("mcpu"), cfg.K, cfg.renorm, cfg.G, cfg.TG, "softmax", cfg.scale, None)
    # softmax in fp32 on either side: ids as sets wherever the oracle's
    # selection margin is wider than a few ulps, weights within 1e-5
    gw, gids, gties, gaps = oracle.grouped_topk(gating.numpy(), cfg.K, cfg.renorm, cfg.G, cfg.TG, "softmax",
                                                cfg.scale, None, exp_mode=oracle.EXP_CR)
    got, want = np.sort(ids.cpu().numpy(), 1), np.sort(gids, 1)
    bad = np.nonzero((got != want).any(1))[0]
    assert len(bad) <= 2, bad
    ok = np.setdiff1d(np.arange(cfg.T), bad)
    a = np.take_along_axis(w.cpu().numpy()[ok], np.argsort(ids.cpu().numpy()[ok], 1), 1)
    b = np.take_along_axis(gw[ok], np.argsort(gids[ok], 1), 1)
    np.testing.assert_allclose(a, b, rtol=1e-5, atol=1e-7)


def test_vllm_native_silu_and_mul_chain_is_bit_exact(mcpu):
    x = C.silu_inputs(64, 1024)
    d = 1024
    xm = x.to("mcpu")
    out = (torch.nn.functional.silu(xm[:, :d]) * xm[:, d:]).cpu()
    bits = out.view(torch.int16).numpy().view(np.uint16)
    want = oracle.silu_and_mul_bf16(x.view(torch.int16).numpy().view(np.uint16), exp_mode=oracle.EXP_CR)
    np.testing.assert_array_equal(bits, want)


def test_vllm_native_rms_norm_chain(mcpu):
    x, w = C.rms_inputs(32, 4096)
    xm, wm = x.to("mcpu"), w.to("mcpu")
    xf = xm.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    y = (xf * torch.rsqrt(var + 1e-6)).to(torch.bfloat16) * wm
    got = y.cpu().float()
    want = torch.from_numpy(oracle.rms_norm_bf16(x.view(torch.int16).numpy().view(np.uint16),
                                                 w.view(torch.int16).numpy().view(np.uint16), 1e-6).view(np.int16)
                            ).view(torch.bfloat16).float()
    # the mean is an fp32 sum here (fp64 in the oracle): at most one bf16 ulp
    torch.testing.assert_close(got, want, rtol=2 ** -7, atol=0)


def test_generic_ops_match_torch_cpu(mcpu):
    g = torch.Generator().manual_seed(3)
    a = torch.randn(7, 5, generator=g)
    b = torch.randn(5, generator=g)
    am, bm = a.to("mcpu"), b.to("mcpu")
    assert torch.equal((am + bm).cpu(), a + b)
    assert torch.equal((am - 2 * bm).cpu(), a - 2 * b)
    assert torch.equal(torch.sub(am, bm, alpha=3).cpu(), torch.sub(a, b, alpha=3))
    assert torch.equal((am * bm).cpu(), a * b)
    assert torch.equal((am / bm).cpu(), a / b)
    assert torch.equal((am + 1.5).cpu(), a + 1.5)
    assert torch.equal((am * 2.5).cpu(), a * 2.5)
    torch.testing.assert_close(torch.rsqrt(am * am + 1).cpu(), torch.rsqrt(a * a + 1), rtol=2e-7, atol=0)
    assert torch.equal(am.pow(2).cpu(), a.pow(2))
    assert torch.equal((-am).cpu(), -a)
    assert torch.equal(am.abs().cpu(), a.abs())
    i = torch.randint(-50, 50, (6, 4), generator=g)
    im = i.to("mcpu")
    assert torch.equal((im + im).cpu(), i + i)
    assert torch.equal((im * 3).cpu(), i * 3)
    assert torch.equal((im / 4).cpu(), i / 4)
    m = torch.rand(7, 5, generator=g) > 0.5
    assert torch.equal((~m.to("mcpu")).cpu(), ~m)
    c = a.clone()
    cm = am.clone()
    c.masked_fill_(m, -7.0)
    cm.masked_fill_(m.to("mcpu"), -7.0)
    assert torch.equal(cm.cpu(), c)
    vals, idx = am.max(dim=1)
    rv, ri = a.max(dim=1)
    assert torch.equal(vals.cpu(), rv) and torch.equal(idx.cpu(), ri)
    vals, idx = am.min(dim=0)
    rv, ri = a.min(dim=0)
    assert torch.equal(vals.cpu(), rv) and torch.equal(idx.cpu(), ri)
    torch.testing.assert_close(am.sum(dim=1).cpu(), a.sum(dim=1), rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(am.mean(dim=0).cpu(), a.mean(dim=0), rtol=1e-6, atol=1e-6)
    tv, ti = am.topk(3, dim=1)
    rv, ri = a.topk(3, dim=1)
    assert torch.equal(tv.cpu(), rv) and torch.equal(ti.cpu(), ri)
    tv, ti = am.topk(2, dim=0, largest=False)
    rv, ri = a.topk(2, dim=0, largest=False)
    assert torch.equal(tv.cpu(), rv) and torch.equal(ti.cpu(), ri)
    torch.testing.assert_close(torch.softmax(am, dim=1).cpu(), torch.softmax(a, dim=1), rtol=2e-6, atol=1e-7)
    torch.testing.assert_close(torch.log_softmax(am, dim=0).cpu(), torch.log_softmax(a, dim=0), rtol=1e-5,
                               atol=1e-6)
    ix = torch.randint(0, 5, (7, 3), generator=g)
    assert torch.equal(am.gather(1, ix.to("mcpu")).cpu(), a.gather(1, ix))
    z = torch.zeros(7, 5)
    zm = z.to("mcpu")
    z.scatter_(1, ix, 2.0)
    zm.scatter_(1, ix.to("mcpu"), 2.0)
    assert torch.equal(zm.cpu(), z)


def test_topk_ties_go_to_the_lower_index(mcpu):
    x = torch.zeros(2, 16)
    x[1, 5] = 1.0
    v, i = x.to("mcpu").topk(4, dim=1)
    assert i.cpu().tolist() == [[0, 1, 2, 3], [5, 0, 1, 2]]
