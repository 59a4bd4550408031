"""The tensor-parallel gated MLP on the B200 against the reference's
fixtures, the oracle and a PyTorch fp32 pipeline.  Tolerance: relative
Frobenius error <= 2e-2 (bf16)."""

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


def bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b)


def tp_forward(cfg, tp, rows=None):
    """Sum of the per-rank partial outputs, computed on one GPU (the
    all-reduce itself is exercised by the multi-GPU bench and tests)."""
    from torch_mcpu_b200.mlp import TPShardSwiGLU

    acc = None
    x_full = None
    for r in range(tp):
        x, rms_w, wgu, wd = C.mlp_weights(cfg, tp, r)
        if rows is not None:
            x = x[rows]
        x_full = x
        shard = TPShardSwiGLU(wgu.to(DEV), wd.to(DEV), None if rms_w is None else rms_w.to(DEV))
        y = shard(x.to(DEV)).float()
        acc = y if acc is None else acc + y
    torch.cuda.synchronize()
    return acc.to(torch.bfloat16), x_full


@pytest.mark.parametrize("name", list(MANIFEST["mlp"]))
def test_mlp_matches_reference_fixture_and_oracle(name):
    e = MANIFEST["mlp"][name]
    cfg = C.MlpCfg(**e["cfg"])
    tp = e["tp"]
    out, _ = tp_forward(cfg, tp)
    gold = oracle.bf16_bits_to_f32(np.load(os.path.join(GOLDEN, e["file"]))["out_bits"].view(np.uint16))
    assert rel(out.float().cpu().numpy(), gold) < 2e-2
    shards = [C.mlp_weights(cfg, tp, r) for r in range(tp)]
    ob = oracle.tp_mlp_bf16(bits(shards[0][0]), [bits(s[2]) for s in shards], [bits(s[3]) for s in shards],
                            None if shards[0][1] is None else bits(shards[0][1]), C.RMS_EPS,
                            exp_mode=oracle.EXP_CR)
    assert rel(out.float().cpu().numpy(), oracle.bf16_bits_to_f32(ob)) < 2e-2


@pytest.mark.parametrize("cfg,tp", [(C.MLP_M1, 1), (C.MLP_M1, 4)]
                         + [(C.MLP_M2_LARGE, tp) for tp in (1, 2, 4, 8)]
                         + [(C.MLP_M2_SMALL, tp) for tp in (1, 2, 4, 8)],
                         ids=lambda v: v.name if isinstance(v, C.MlpCfg) else f"tp{v}")
def test_mlp_full_shape_matches_fp32_pipeline(cfg, tp):
    """Full weights at the benchmark shapes (the TP example's gated MLP, and
    the pre-rms_norm SwiGLU block H=7168 / I=18432 at 8192 and 256 tokens),
    every rank's shard run on one GPU and the partials summed; the fp32
    reference is evaluated on 64 sampled rows."""
    from torch_mcpu_b200 import device_error

    device_error(reset=True)
    out, x = tp_forward(cfg, tp)
    assert device_error() == 0
    rows = torch.arange(0, cfg.T, max(1, cfg.T // 64))
    ref = None
    for r in range(tp):
        x_r, rms_w, wgu, wd = C.mlp_weights(cfg, tp, r)
        h = x_r[rows].to(DEV).float()
        if rms_w is not None:
            var = h.pow(2).mean(-1, keepdim=True)
            h = (h * torch.rsqrt(var + C.RMS_EPS)).to(torch.bfloat16).float() * rms_w.to(DEV).float()
            h = h.to(torch.bfloat16).float()
        gu = (h @ wgu.to(DEV).float().t()).to(torch.bfloat16).float()
        I = gu.shape[1] // 2
        a = (torch.nn.functional.silu(gu[:, :I]).to(torch.bfloat16).float() * gu[:, I:]).to(torch.bfloat16)
        y = a.float() @ wd.to(DEV).float().t()
        ref = y if ref is None else ref + y
    got = out[rows.to(DEV)].float()
    assert rel(got.cpu().numpy(), ref.cpu().numpy()) < 2e-2
