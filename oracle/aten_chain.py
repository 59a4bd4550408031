"""The reference's mcpu path, op by op, on the host cores.

TEST INFRASTRUCTURE ONLY: bench.py's CPU legs and tests/ use it as the
timed baseline of the reference's CPU implementation.

On the reference's mcpu device every aten op of these chains dispatches to a
csrc/aten/ops/*.cpp kernel that runs PyTorch's CPU ATen kernel on a host view
of the tensor (e.g. topk.cpp:10-40, binary_out.cpp:189-229), except sigmoid
and silu, which are scalar loops on one worker thread
(unary_out.cpp:46-61, raw_unary_value), and pow / rsqrt, which take the CPU
fallback.  The restatements below run the same sequence of ATen CPU kernels
on CPU tensors and the raw loops through the C oracle (glibc expf, one
thread), so their cost is the reference's arithmetic without its launch
queue, host-view copies and fallback synchronisations.

  grouped_topk_chain   tests/test_grouped_topk_compile.py:28-66
  silu_and_mul_chain   F.silu(x[:, :d]) * x[:, d:] (vLLM SiluAndMul native)
  rms_norm_chain       (x.float() * rsqrt(mean(x.float()^2) + eps)).to(bf16) * w
  gated_mlp_chain      mm -> silu -> mul -> mm of example/01_mlp_tp4/run.py:50-56
                       in its SwiGLU form (one rank, TP=1)
"""

from __future__ import annotations

import numpy as np
import torch

from . import EXP_GLIBC, sigmoid_f32, silu_raw_bf16


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _from_bits(b: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16)


def grouped_topk_chain(gating: torch.Tensor, topk: int, renormalize: bool, num_expert_group: int,
                       topk_group: int, scoring_func: str = "softmax", routed_scaling_factor: float = 1.0,
                       e_score_correction_bias: torch.Tensor | None = None):
    """The router's op sequence (test_grouped_topk_compile.py:28-66) on CPU
    fp32 tensors; returns (weights fp32 [T, topk], ids int32 [T, topk])."""
    T, E = gating.shape
    G = num_expert_group
    if scoring_func == "sigmoid":   # raw loop, one thread (unary_out.cpp:46-49)
        scores = torch.from_numpy(sigmoid_f32(gating.numpy(), EXP_GLIBC))
    else:                           # _softmax_out (softmax_random_argmax.cpp:57-82)
        scores = torch.softmax(gating, dim=-1)
    if e_score_correction_bias is not None:
        unbiased = scores
        scores = scores + e_score_correction_bias.unsqueeze(0)                 # add.Tensor
        top2 = scores.view(T, G, -1).topk(2, dim=-1)[0]                         # topk.values
        group_scores = top2.sum(dim=-1)                                         # sum.IntList_out
    else:
        group_scores = scores.view(T, G, -1).max(dim=-1).values                 # max.dim_max
    picked = torch.topk(group_scores, k=topk_group, dim=-1, sorted=False)[1]
    group_mask = torch.zeros_like(group_scores)                                 # zero_
    group_mask.scatter_(1, picked, 1)                                           # scatter.value (fallback)
    expert_mask = group_mask.unsqueeze(-1).expand(T, G, E // G).reshape(T, -1)  # copy
    masked = scores.masked_fill(~expert_mask.bool(), float("-inf"))             # bitwise_not, masked_fill_
    if e_score_correction_bias is not None:
        ids = torch.topk(masked, k=topk, dim=-1, sorted=False)[1]
        weights = unbiased.gather(1, ids)                                       # gather.out
    else:
        weights, ids = torch.topk(masked, k=topk, dim=-1, sorted=False)
    if renormalize:
        weights = weights / weights.sum(dim=-1, keepdim=True)                   # sum, div
    if routed_scaling_factor != 1.0:
        weights = weights * routed_scaling_factor                               # mul
    return weights.to(torch.float32), ids.to(torch.int32)


def silu_and_mul_chain(x: torch.Tensor) -> torch.Tensor:
    """x bf16 [T, 2d] -> bf16 [T, d]: the raw silu loop on x[:, :d] (one
    thread, rounded to bf16), then the aten mul in bf16."""
    d = x.shape[-1] // 2
    a = _from_bits(silu_raw_bf16(_bits(x), d, EXP_GLIBC))
    return a * x[:, d:]


def rms_norm_chain(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """vLLM's native rms_norm as the mcpu device runs it op by op (pow and
    rsqrt through the CPU fallback, mean through reduction_scatter.cpp)."""
    xf = x.float()
    var = xf.pow(2).mean(dim=-1, keepdim=True)
    return (xf * torch.rsqrt(var + eps)).to(torch.bfloat16) * w


def gated_mlp_chain(x: torch.Tensor, w_gate_up: torch.Tensor, w_down: torch.Tensor) -> torch.Tensor:
    """One TP=1 step of the gated MLP in bf16: mm (oneDNN, as mm.cpp:13-43
    calls at::mm_out), the raw silu loop, mul, mm."""
    gu = torch.mm(x, w_gate_up.t())
    inter = gu.shape[1] // 2
    a = silu_and_mul_chain(gu.contiguous()) if inter > 0 else gu
    return torch.mm(a, w_down.t())
