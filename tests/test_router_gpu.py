"""grouped_topk on the B200 against the oracle and the reference's fixtures.

Parity bar: topk_ids bit-exact as per-row sets (the reference's own order is
an ATen artefact), topk_weights matched by id within 1e-6 relative (fp32
logits) or within one bf16 ulp, 2^-8 relative (bf16 logits: the reference
rounds the scores, the renormalisation sum and the weights to bf16, and the
GPU rounds at the same points; only the order of the eight-term sum, which
the reference takes in its own topk output order, can move a weight by one
ulp).  The oracle itself matches the reference's bf16 fixtures bit for bit.
Every call goes through the C-ABI entry point mcpu_grouped_topk.
"""

import hashlib
import json
import os

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))
DEV = "cuda:0"
BF16_ULP = 2.0 ** -8


def _mcpu():
    import torch_mcpu_b200

    return torch_mcpu_b200


def _by_id(w, ids):
    o = np.argsort(ids, axis=1, kind="stable")
    return np.take_along_axis(w, o, 1), np.take_along_axis(ids, o, 1)


def _gpu(cfg, gating, bias):
    m = _mcpu()
    g = gating.to(DEV)
    b = None if bias is None else bias.to(DEV)
    w, ids = m.grouped_topk(torch.empty(g.shape[0], 1, device=DEV), g, cfg.K, cfg.renorm, cfg.G,
                            cfg.TG, cfg.scoring, cfg.scale, b)
    torch.cuda.synchronize()
    assert w.dtype == torch.float32 and ids.dtype == torch.int32
    return w.cpu().numpy(), ids.cpu().numpy()


def _oracle(cfg, gating, bias, mode=oracle.EXP_CR):
    g = gating.view(torch.int16).numpy().view(np.uint16) if gating.dtype == torch.bfloat16 else gating.numpy()
    return oracle.grouped_topk(g, cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring, cfg.scale,
                               None if bias is None else bias.numpy(), exp_mode=mode)


def _assert_parity(cfg, w, ids, ow, oids, oties, rtol):
    ws, idss = _by_id(w, ids)
    ows, oidss = _by_id(ow, oids)
    np.testing.assert_array_equal(idss, oidss)
    np.testing.assert_allclose(ws, ows, rtol=rtol, atol=0)
    # ids within a row are distinct
    assert (np.diff(idss, axis=1) > 0).all()


@pytest.mark.parametrize("cfg", C.ROUTER_GOLDEN, ids=lambda c: c.name)
def test_router_matches_oracle_and_reference(cfg):
    gating, bias = C.router_inputs(cfg)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    rtol = 1e-6 if cfg.dtype == "float32" else BF16_ULP
    _assert_parity(cfg, w, ids, ow, oids, oties, rtol)
    fx = np.load(os.path.join(GOLDEN, f"router_{cfg.name}.npz"))
    ok = ~fx["ambiguous"]
    ws, idss = _by_id(w, ids)
    np.testing.assert_array_equal(idss[ok], fx["ids_sorted"][ok].astype(np.int32))
    np.testing.assert_allclose(ws[ok], fx["weights_by_id"][ok], rtol=1e-5 if cfg.dtype == "float32" else BF16_ULP)


@pytest.mark.parametrize("cfg", C.ROUTER_LARGE, ids=lambda c: c.name)
def test_router_full_size_matches_oracle_and_reference_digest(cfg):
    m = _mcpu()
    gating, bias = C.router_inputs(cfg)
    m.grouped_topk_exact_rows(reset=True)
    w, ids = _gpu(cfg, gating, bias)
    exact_rows = m.grouped_topk_exact_rows()
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    _assert_parity(cfg, w, ids, ow, oids, oties, 1e-6)
    entry = MANIFEST["router"][cfg.name]
    fx = np.load(os.path.join(GOLDEN, entry["file"]))
    amb = fx["ambiguous"]
    ws, idss = _by_id(w, ids)
    h = hashlib.sha256(np.ascontiguousarray(idss[~amb].astype(np.int32)).tobytes()).hexdigest()
    assert h == entry["ids_sorted_sha256"]
    np.testing.assert_allclose(ws[fx["rows"]], fx["weights_by_id"], rtol=1e-5)
    if cfg.scoring == "sigmoid" and cfg.bias:
        # the near-tie path ran and is part of what was just checked
        assert 0 < exact_rows < cfg.T // 20


def test_reference_regression_case_bf16_softmax():
    """tests/test_grouped_topk_compile.py:79-100 of the reference."""
    fx = np.load(os.path.join(GOLDEN, "router_reference_test_8x16_bf16.npz"))
    hidden, gating = C.reference_test_inputs()
    a = C.REFERENCE_TEST_ARGS
    w, ids = _mcpu().grouped_topk(hidden.to(DEV), gating.to(DEV), **a)
    ws, idss = _by_id(w.cpu().numpy(), ids.cpu().numpy())
    ok = ~fx["ambiguous"]
    np.testing.assert_array_equal(idss[ok], fx["ids_sorted"][ok].astype(np.int32))
    np.testing.assert_allclose(ws[ok], fx["weights_by_id"][ok], rtol=BF16_ULP)


EDGE = [
    C.RouterCfg("ragged_T1000", 1000, 256, 8, 4, 8, "sigmoid", True, True, 2.5),
    C.RouterCfg("ragged_T33_noscale", 33, 256, 8, 4, 8, "sigmoid", True, False, 1.0),
    C.RouterCfg("G32_GS8", 300, 256, 32, 4, 8, "sigmoid", True, True, 1.0),
    C.RouterCfg("G1_E64", 200, 64, 1, 1, 8, "softmax", False, True, 1.0),
    C.RouterCfg("G4_K16", 200, 128, 4, 2, 16, "sigmoid", True, True, 2.0),
    C.RouterCfg("sigmoid_nobias", 500, 256, 8, 4, 8, "sigmoid", False, True, 2.5),
    C.RouterCfg("softmax_bias", 500, 256, 8, 4, 8, "softmax", True, True, 1.0),
    C.RouterCfg("odd_group_20", 129, 160, 8, 3, 6, "softmax", False, False, 1.0),
    C.RouterCfg("bf16_odd", 77, 160, 8, 3, 6, "sigmoid", True, True, 2.5, "bfloat16"),
    C.RouterCfg("K_equals_candidates", 64, 64, 8, 1, 8, "sigmoid", True, True, 1.0),
]


@pytest.mark.parametrize("cfg", EDGE, ids=lambda c: c.name)
def test_router_edge_configurations(cfg):
    gating, bias = C.router_inputs(cfg)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    if cfg.scoring == "softmax" and cfg.bias:
        # softmax + bias ranks on the GPU's own fp32 softmax; rows whose
        # boundary gap is below a few ulp may resolve differently
        _, _, _, gaps = _oracle(cfg, gating, bias)
        keep = gaps > 1e-5
        ws, idss = _by_id(w, ids)
        ows, oidss = _by_id(ow, oids)
        np.testing.assert_array_equal(idss[keep], oidss[keep])
        np.testing.assert_allclose(ws[keep], ows[keep], rtol=1e-5)
        return
    rtol = 1e-6 if cfg.dtype == "float32" else BF16_ULP
    _assert_parity(cfg, w, ids, ow, oids, oties, rtol)


KERNEL_CASES = [C.deepseek_v3(t) for t in (1, 16, 33, 256, 1000, 4096, 65536)] + [
    C.RouterCfg("TG2_K4", 777, 256, 8, 2, 4, "sigmoid", True, True, 1.0),
    C.RouterCfg("TG3_K6_noscale", 515, 256, 8, 3, 6, "sigmoid", True, False, 2.5),
    C.RouterCfg("TG4_K5", 300, 256, 8, 4, 5, "sigmoid", True, True, 2.5),
    C.RouterCfg("TG1_K2", 64, 256, 8, 1, 2, "sigmoid", True, True, 1.0),
]


@pytest.mark.parametrize("kernel", ["lanes4", "pair", "quad"])
@pytest.mark.parametrize("cfg", KERNEL_CASES, ids=lambda c: c.name)
def test_router_pair_and_quad_kernels_at_every_size(cfg, kernel, monkeypatch):
    """The DeepSeek-V3 shape (256 experts, 8 groups, fp32, sigmoid + bias) is
    served by the four-lane kernel (topk_group 4, topk 8), the pair kernel
    (two lanes per token, other topk_group / topk, from 8192 tokens) or the
    first quad kernel (below 8192 tokens); each is forced here over
    ragged, tiny and full-size batches and other topk_group / topk choices."""
    monkeypatch.setenv("MCPU_ROUTER_KERNEL", kernel)
    gating, bias = C.router_inputs(cfg)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    _assert_parity(cfg, w, ids, ow, oids, oties, 1e-6)


@pytest.mark.parametrize("kernel", ["lanes4", "pair", "quad"])
def test_router_many_equal_keys_take_the_exact_paths(kernel, monkeypatch):
    """Rows whose keys tie in many places: all keys equal (every group and
    expert margin is zero), and rows where a whole group ties, so the
    candidate lists are long and both exact paths (group re-pick, exact
    re-rank) run."""
    monkeypatch.setenv("MCPU_ROUTER_KERNEL", kernel)
    cfg = C.RouterCfg("ties_many", 96, 256, 8, 4, 8, "sigmoid", True, True, 2.5)
    g = torch.Generator().manual_seed(4)
    gating = torch.randn(96, 256, generator=g)
    gating[0::3] = 0.0                      # every key equal
    gating[1::3, 64:96] = 3.0               # group 2 ties at the top
    gating[2::3, :] = torch.randn(1, 256, generator=g).round()  # coarse values, many equal keys
    bias = torch.zeros(256)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    _assert_parity(cfg, w, ids, ow, oids, oties, 1e-6)


def test_router_exact_ties_break_toward_lower_index():
    cfg = C.RouterCfg("ties", 40, 256, 8, 4, 8, "sigmoid", True, True, 2.5)
    gating = torch.zeros(40, 256)
    gating[1::2, 37] = 1.0  # break some ties only in odd rows
    bias = torch.zeros(256)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    np.testing.assert_array_equal(ids, oids)  # same order too: exact path
    np.testing.assert_array_equal(ids[0], np.arange(8))
    np.testing.assert_allclose(w, ow, rtol=1e-6)


def test_router_empty_and_single_token():
    m = _mcpu()
    g = torch.empty(0, 256, device=DEV)
    w, ids = m.grouped_topk(g, g, 8, True, 8, 4, "sigmoid", 2.5, torch.zeros(256, device=DEV))
    assert w.shape == (0, 8) and ids.shape == (0, 8)
    cfg = C.deepseek_v3(1)
    gating, bias = C.router_inputs(cfg)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    _assert_parity(cfg, w, ids, ow, oids, oties, 1e-6)


def test_router_non_contiguous_and_misaligned_inputs():
    cfg = C.deepseek_v3(256)
    gating, bias = C.router_inputs(cfg)
    m = _mcpu()
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    # a strided view (copied to contiguous by the op)
    big = torch.zeros(256, 512, device=DEV)
    big[:, 1:257] = gating.to(DEV)
    w, ids = m.grouped_topk(big, big[:, 1:257], 8, True, 8, 4, "sigmoid", 2.5, bias.to(DEV))
    _assert_parity(cfg, w.cpu().numpy(), ids.cpu().numpy(), ow, oids, oties, 1e-6)
    # a contiguous tensor 4 bytes off a 16-byte boundary: scalar-load path
    flat = torch.zeros(1 + gating.numel(), device=DEV)
    g = flat[1:].view(256, 256)
    g.copy_(gating.to(DEV))
    w, ids = m.grouped_topk(g, g, 8, True, 8, 4, "sigmoid", 2.5, bias.to(DEV))
    _assert_parity(cfg, w.cpu().numpy(), ids.cpu().numpy(), ow, oids, oties, 1e-6)


def test_router_rejects_bad_arguments_like_the_reference():
    m = _mcpu()
    g = torch.zeros(4, 12, device=DEV)
    with pytest.raises(RuntimeError, match="divisible"):
        m.grouped_topk(g, g, 2, True, 8, 1, "softmax")
    with pytest.raises(RuntimeError, match="exceeds"):
        m.grouped_topk(g, torch.zeros(4, 16, device=DEV), 9, True, 4, 2, "softmax")
    with pytest.raises(ValueError, match="Unsupported scoring"):
        m.grouped_topk(g, g, 2, True, 4, 1, "relu")
    with pytest.raises(AssertionError):
        m.grouped_topk(torch.zeros(3, 1, device=DEV), g, 2, True, 4, 1, "softmax")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        m.grouped_topk(torch.zeros(4, 1), torch.zeros(4, 16), 2, True, 4, 2, "softmax")


def test_router_is_stream_ordered():
    """The op enqueues on the current stream and returns before completion."""
    m = _mcpu()
    cfg = C.deepseek_v3(4096)
    gating, bias = C.router_inputs(cfg)
    s = torch.cuda.Stream()
    g, b = gating.to(DEV), bias.to(DEV)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        w, ids = m.grouped_topk(g, g, 8, True, 8, 4, "sigmoid", 2.5, b)
    s.synchronize()
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    _assert_parity(cfg, w.cpu().numpy(), ids.cpu().numpy(), ow, oids, oties, 1e-6)


PATH_CASES = [
    # (config, env) -- which kernel serves it is decided by the host dispatch
    (C.RouterCfg("generic_tma_G2", 300, 64, 2, 1, 4, "sigmoid", True, True, 1.0), {}),
    (C.RouterCfg("direct_E512", 200, 512, 8, 4, 8, "sigmoid", True, True, 2.5), {}),
    (C.deepseek_v3(4096), {"MCPU_ROUTER_NO_TMA": "1"}),
    (C.softmax160(777), {"MCPU_ROUTER_NO_TMA": "1"}),
    (C.RouterCfg("all_groups_G4", 500, 128, 4, 4, 8, "sigmoid", True, True, 2.5), {}),
    (C.RouterCfg("single_group_E64", 300, 64, 1, 1, 6, "softmax", False, True, 1.0), {}),
]


@pytest.mark.parametrize("cfg,env", PATH_CASES, ids=lambda v: v.name if hasattr(v, "name") else str(v))
def test_router_every_kernel_path(cfg, env, monkeypatch):
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    gating, bias = C.router_inputs(cfg)
    w, ids = _gpu(cfg, gating, bias)
    ow, oids, oties, _ = _oracle(cfg, gating, bias)
    _assert_parity(cfg, w, ids, ow, oids, oties, 1e-6)


def test_router_repeated_calls_reuse_the_stream_worklist():
    """The exact kernel resets the per-stream worklist after each call."""
    m = _mcpu()
    cfg = C.deepseek_v3(65536)
    gating, bias = C.router_inputs(cfg)
    g, b = gating.to(DEV), bias.to(DEV)
    outs = [m.grouped_topk(g, g, 8, True, 8, 4, "sigmoid", 2.5, b) for _ in range(3)]
    torch.cuda.synchronize()
    for w, ids in outs[1:]:
        assert torch.equal(ids, outs[0][1]) and torch.equal(w, outs[0][0])
    assert m.device_error() == 0
