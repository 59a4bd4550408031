"""The oracle pinned against the reference's own outputs (golden fixtures).

CPU only.  The fixtures were produced by tests/golden/gen_golden.py from the
reference's router function and vLLM's native formulas; see that script.
"""

import json
import os

import numpy as np
import pytest
import torch

import oracle
import configs as C

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
MANIFEST = json.load(open(os.path.join(GOLDEN, "manifest.json")))


def _np_inputs(cfg):
    gating, bias = C.router_inputs(cfg)
    if gating.dtype == torch.bfloat16:
        g = gating.view(torch.int16).numpy().view(np.uint16)
    else:
        g = gating.numpy()
    return g, (None if bias is None else bias.numpy())


def _run_oracle(cfg, exp_mode=oracle.EXP_GLIBC):
    g, b = _np_inputs(cfg)
    return oracle.grouped_topk(g, cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring, cfg.scale, b,
                               exp_mode=exp_mode)


def _by_id(w, ids):
    o = np.argsort(ids, axis=1, kind="stable")
    return np.take_along_axis(w, o, 1), np.take_along_axis(ids, o, 1)


@pytest.mark.parametrize("cfg", C.ROUTER_GOLDEN, ids=lambda c: c.name)
def test_router_oracle_matches_reference(cfg):
    fx = np.load(os.path.join(GOLDEN, f"router_{cfg.name}.npz"))
    w, ids, ties, _ = _run_oracle(cfg)
    ws, idss = _by_id(w, ids)
    amb = fx["ambiguous"]
    ok = ~amb
    np.testing.assert_array_equal(idss[ok], fx["ids_sorted"][ok].astype(np.int32))
    # weights matched by expert id; 1e-5 relative for fp32, bit for bit for
    # bf16 inputs (the oracle rounds to bf16 where the reference's aten chain
    # rounds)
    rtol = 1e-5 if cfg.dtype == "float32" else 0.0
    np.testing.assert_allclose(ws[ok], fx["weights_by_id"][ok], rtol=rtol, atol=0)
    assert not ties[ok].any()


@pytest.mark.parametrize("cfg", C.ROUTER_LARGE, ids=lambda c: c.name)
def test_router_oracle_matches_reference_large(cfg):
    entry = MANIFEST["router"][cfg.name]
    fx = np.load(os.path.join(GOLDEN, entry["file"]))
    w, ids, ties, _ = _run_oracle(cfg)
    ws, idss = _by_id(w, ids)
    amb = fx["ambiguous"]
    import hashlib

    h = hashlib.sha256(np.ascontiguousarray(idss[~amb].astype(np.int32)).tobytes()).hexdigest()
    assert h == entry["ids_sorted_sha256"]
    rows = fx["rows"]
    np.testing.assert_allclose(ws[rows], fx["weights_by_id"], rtol=1e-5, atol=0)
    # the oracle's own tie flag marks every row the reference found ambiguous
    # or leaves it unflagged only when the logit order resolves it
    assert ties.sum() <= max(1, amb.sum())


def test_router_reference_regression_case():
    """tests/test_grouped_topk_compile.py:79-100 (8x16 bf16 softmax)."""
    fx = np.load(os.path.join(GOLDEN, "router_reference_test_8x16_bf16.npz"))
    _, gating = C.reference_test_inputs()
    a = C.REFERENCE_TEST_ARGS
    w, ids, _, _ = oracle.grouped_topk(gating.view(torch.int16).numpy().view(np.uint16), a["topk"],
                                       a["renormalize"], a["num_expert_group"], a["topk_group"],
                                       a["scoring_func"], a["routed_scaling_factor"], None)
    ws, idss = _by_id(w, ids)
    ok = ~fx["ambiguous"]
    np.testing.assert_array_equal(idss[ok], fx["ids_sorted"][ok].astype(np.int32))
    np.testing.assert_allclose(ws[ok], fx["weights_by_id"][ok], rtol=0.0)


def test_glibc_and_correctly_rounded_exp_agree_on_fixtures():
    """The CUDA exact path rounds exp correctly; the reference uses glibc
    expf.  On every fixture configuration the two give the same ids."""
    for cfg in C.ROUTER_GOLDEN + C.ROUTER_LARGE:
        if cfg.scoring != "sigmoid":
            continue
        w0, i0, _, _ = _run_oracle(cfg, oracle.EXP_GLIBC)
        w1, i1, _, _ = _run_oracle(cfg, oracle.EXP_CR)
        np.testing.assert_array_equal(i0, i1)
        np.testing.assert_allclose(w0, w1, rtol=2e-7)


def test_sigmoid_restates_raw_loop():
    x = np.linspace(-30, 30, 10001, dtype=np.float32)
    s = oracle.sigmoid_f32(x)
    ref = (np.float32(1.0) / (np.float32(1.0) + np.exp(-x.astype(np.float64)).astype(np.float32)))
    np.testing.assert_allclose(s, ref, rtol=3e-7)


def _bf16_ulp_diff(a_bits, b_bits):
    a = a_bits.astype(np.int32)
    b = b_bits.astype(np.int32)
    # map sign-magnitude to a monotone integer line
    a = np.where(a & 0x8000, -(a & 0x7FFF), a)
    b = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(a - b)


@pytest.mark.parametrize("name", [k for k in MANIFEST["bandwidth"] if k.startswith("silu")])
def test_silu_and_mul_oracle_matches_vllm(name):
    e = MANIFEST["bandwidth"][name]
    x = C.silu_inputs(e["T"], e["d"])
    out = oracle.silu_and_mul_bf16(x.view(torch.int16).numpy().view(np.uint16))
    gold = np.load(os.path.join(GOLDEN, e["file"]))["out_bits"].view(np.uint16)
    d = _bf16_ulp_diff(out, gold)
    assert d.max() <= 1 and (d > 0).mean() < 2e-3


@pytest.mark.parametrize("name", [k for k in MANIFEST["bandwidth"] if k.startswith("rms")])
def test_rms_norm_oracle_matches_vllm(name):
    e = MANIFEST["bandwidth"][name]
    x, w = C.rms_inputs(e["T"], e["H"])
    out = oracle.rms_norm_bf16(x.view(torch.int16).numpy().view(np.uint16),
                               w.view(torch.int16).numpy().view(np.uint16), e["eps"])
    gold = np.load(os.path.join(GOLDEN, e["file"]))["out_bits"].view(np.uint16)
    d = _bf16_ulp_diff(out, gold)
    assert d.max() <= 1 and (d > 0).mean() < 2e-3


@pytest.mark.parametrize("name", list(MANIFEST["mlp"]))
def test_mlp_oracle_matches_reference_structure(name):
    e = MANIFEST["mlp"][name]
    cfg = C.MlpCfg(**e["cfg"])
    tp = e["tp"]
    shards = [C.mlp_weights(cfg, tp, r) for r in range(tp)]
    x, rms_w = shards[0][0], shards[0][1]
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    out = oracle.tp_mlp_bf16(bits(x), [bits(s[2]) for s in shards], [bits(s[3]) for s in shards],
                             None if rms_w is None else bits(rms_w), C.RMS_EPS)
    gold = np.load(os.path.join(GOLDEN, e["file"]))["out_bits"].view(np.uint16)
    a = oracle.bf16_bits_to_f32(out).astype(np.float64)
    b = oracle.bf16_bits_to_f32(gold).astype(np.float64)
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    assert rel < 2e-2, rel


def test_oracle_rejects_bad_arguments():
    g = np.zeros((2, 10), np.float32)
    with pytest.raises(ValueError):
        oracle.grouped_topk(g, 2, True, 3, 1, "softmax")  # 10 % 3 != 0
    with pytest.raises(ValueError):
        oracle.grouped_topk(g, 9, True, 5, 1, "softmax")  # k > topk_group * group size


@pytest.mark.parametrize("cfg", [c for c in C.ROUTER_GOLDEN if c.dtype == "float32"], ids=lambda c: c.name)
def test_router_op_chain_restatement_matches_reference_fixtures(cfg):
    """oracle/aten_chain.py (the reference's router op by op, timed as the
    CPU baseline) gives the reference fixtures' ids and weights."""
    from oracle import aten_chain

    fx = np.load(os.path.join(GOLDEN, f"router_{cfg.name}.npz"))
    gating, bias = C.router_inputs(cfg)
    w, ids = aten_chain.grouped_topk_chain(gating, cfg.K, cfg.renorm, cfg.G, cfg.TG, cfg.scoring, cfg.scale,
                                           bias)
    ws, idss = _by_id(w.numpy(), ids.numpy())
    ok = ~fx["ambiguous"]
    np.testing.assert_array_equal(idss[ok], fx["ids_sorted"][ok].astype(np.int32))
    np.testing.assert_allclose(ws[ok], fx["weights_by_id"][ok], rtol=1e-6, atol=0)


def test_silu_and_rms_op_chains_match_the_oracle():
    from oracle import aten_chain

    x = C.silu_inputs(33, 1000)
    got = aten_chain.silu_and_mul_chain(x).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, oracle.silu_and_mul_bf16(x.view(torch.int16).numpy().view(np.uint16)))
    x, w = C.rms_inputs(9, 4096)
    got = aten_chain.rms_norm_chain(x, w, C.RMS_EPS).view(torch.int16).numpy().view(np.uint16)
    want = oracle.rms_norm_bf16(x.view(torch.int16).numpy().view(np.uint16), w.view(torch.int16).numpy().view(np.uint16),
                                C.RMS_EPS)
    assert np.array_equal(got, want)
