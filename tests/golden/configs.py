"""Seeded synthetic inputs for the hot-path configurations.

Shared by the fixture generator (gen_golden.py), the parity tests and
bench.py so that every leg sees the same numbers: all tensors are drawn on
the CPU from ``torch.Generator().manual_seed(seed)`` and only then moved to a
device.  Standard deviations are read as std (N(0, 0.01) -> std 0.01).
"""

from __future__ import annotations

import functools
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class RouterCfg:
    name: str
    T: int
    E: int
    G: int
    TG: int
    K: int
    scoring: str  # "sigmoid" | "softmax"
    bias: bool
    renorm: bool
    scale: float
    dtype: str = "float32"  # gating dtype: float32 | bfloat16
    seed: int = 0


# DeepSeek-V3-style router: 256 experts, 8 groups, top-4 groups, top-8,
# sigmoid scoring with a correction bias, renormalised, x2.5.
def deepseek_v3(T: int, seed: int = 0, dtype: str = "float32") -> RouterCfg:
    return RouterCfg(f"sig_bias_T{T}_E256" + ("" if dtype == "float32" else "_bf16"),
                     T, 256, 8, 4, 8, "sigmoid", True, True, 2.5, dtype, seed)


# Softmax variant: 160 experts, 8 groups, top-3 groups, top-6, no bias.
def softmax160(T: int, renorm: bool = False, seed: int = 0) -> RouterCfg:
    return RouterCfg(f"softmax_T{T}_E160" + ("_renorm" if renorm else ""),
                     T, 160, 8, 3, 6, "softmax", False, renorm, 1.0, "float32", seed)


ROUTER_GOLDEN = [
    deepseek_v3(1),
    deepseek_v3(16),
    deepseek_v3(256),
    deepseek_v3(1024),           # the CPU-runnable headline case (1024 x 256)
    deepseek_v3(4096),
    deepseek_v3(512, dtype="bfloat16"),
    softmax160(1024),
    softmax160(1024, renorm=True),
]

ROUTER_LARGE = [deepseek_v3(65536), softmax160(65536)]


def router_inputs(cfg: RouterCfg):
    """gating [T, E] (fp32 N(0,1), or rounded to bf16) and bias [E] fp32
    N(0, 0.01) drawn from the same generator after the logits."""
    g = torch.Generator().manual_seed(cfg.seed)
    gating = torch.randn(cfg.T, cfg.E, generator=g, dtype=torch.float32)
    bias = torch.randn(cfg.E, generator=g, dtype=torch.float32) * 0.01 if cfg.bias else None
    if cfg.dtype == "bfloat16":
        gating = gating.to(torch.bfloat16)
    return gating, bias


def reference_test_inputs():
    """The reference's own regression case (tests/test_grouped_topk_compile.py:
    69-76): global seed 0, hidden [8,16] then gating [8,16], both bf16."""
    torch.manual_seed(0)
    hidden = torch.randn(8, 16, dtype=torch.bfloat16)
    gating = torch.randn(8, 16, dtype=torch.bfloat16)
    return hidden, gating


REFERENCE_TEST_ARGS = dict(topk=2, renormalize=True, num_expert_group=4, topk_group=2,
                           scoring_func="softmax", routed_scaling_factor=1.0)


# ------------------------------------------------------------- bandwidth ops
def silu_inputs(T: int, d: int, seed: int = 1) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, 2 * d, generator=g, dtype=torch.float32).to(torch.bfloat16)


def rms_inputs(T: int, H: int, seed: int = 2):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g, dtype=torch.float32).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(H, generator=g, dtype=torch.float32)).to(torch.bfloat16)
    return x, w


SILU_FULL = (8192, 18432)   # input [8192, 2 x 18432]
RMS_FULL = (8192, 7168)
RMS_EPS = 1e-6


# ------------------------------------------------------------- gated MLP
@dataclass(frozen=True)
class MlpCfg:
    name: str
    T: int
    H: int
    I: int
    pre_norm: bool
    seed: int = 3


MLP_M1 = MlpCfg("gated_mlp_H4096_I14336_T2048", 2048, 4096, 14336, False)
MLP_M2_SMALL = MlpCfg("swiglu_prenorm_H7168_I18432_T256", 256, 7168, 18432, True)
MLP_M2_LARGE = MlpCfg("swiglu_prenorm_H7168_I18432_T8192", 8192, 7168, 18432, True)


def mlp_weights(cfg: MlpCfg, tp: int, rank: int):
    """Weights of one tensor-parallel rank, identical for every TP degree.

    The intermediate dimension is cut into 8 fixed blocks (8 = the largest TP
    degree); block b of W_gate, W_up and W_down^T is drawn from its own seed,
    so rank r of TP=tp owns blocks [r*8/tp, (r+1)*8/tp) and never builds the
    other ranks' shards.  Returns bf16 tensors:
    x [T, H], rms_w [H] or None, w_gate_up [2*I/tp, H] = [gate_r; up_r]
    (column-parallel rows) and w_down [H, I/tp] (row-parallel columns).
    """
    g = torch.Generator().manual_seed(cfg.seed)
    x = torch.randn(cfg.T, cfg.H, generator=g, dtype=torch.float32).to(torch.bfloat16)
    rms_w = None
    if cfg.pre_norm:
        rms_w = (1.0 + 0.1 * torch.randn(cfg.H, generator=g)).to(torch.bfloat16)
    assert 8 % tp == 0 and cfg.I % 8 == 0
    nb = 8 // tp
    blocks = range(rank * nb, (rank + 1) * nb)
    gate = torch.cat([_block_normal(cfg.seed, 1, b, cfg.I // 8, cfg.H) for b in blocks], 0)
    up = torch.cat([_block_normal(cfg.seed, 2, b, cfg.I // 8, cfg.H) for b in blocks], 0)
    down_t = torch.cat([_block_normal(cfg.seed, 3, b, cfg.I // 8, cfg.H) for b in blocks], 0)
    return x, rms_w, torch.cat([gate, up], 0), down_t.t().contiguous()


@functools.lru_cache(maxsize=None)
def _block_normal(seed: int, which: int, block: int, rows: int, cols: int) -> torch.Tensor:
    """One fixed block of a weight matrix (cached: the TP degrees of one
    configuration share their blocks, and torch.cat copies them out)."""
    g = torch.Generator().manual_seed((seed * 16 + which) * 64 + block)
    return (0.02 * torch.randn(rows, cols, generator=g, dtype=torch.float32)).to(torch.bfloat16)


MLP_TINY = MlpCfg("gated_mlp_H256_I512_T32", 32, 256, 512, False)
MLP_TINY_NORM = MlpCfg("swiglu_prenorm_H256_I1024_T48", 48, 256, 1024, True)
