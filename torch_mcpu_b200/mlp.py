"""Tensor-parallel gated MLP on the mcpu B200 kernels.

The structure of the reference's example/01_mlp_tp4/run.py (TPShardMLP
lines 35-56, run_one_step 106-113): column-parallel up projection,
activation, row-parallel down projection, then one SUM all-reduce of the
partial outputs.  Here in the gated (SwiGLU) form of the benchmark
configurations, optionally preceded by rms_norm:

    h = rms_norm(x)                       (optional, replicated per rank)
    a = silu(h Wg_r^T) * (h Wu_r^T)       one tcgen05 GEMM with fused epilogue
    y_r = a Wd_r^T                        tcgen05 GEMM
    y = all_reduce(sum_r y_r)             NCCL over NVLink (torch.distributed)

or, on mcpu tensors with a symmetric window (mcpu_tp_step), the last two
lines as one kernel that sends the partial tiles over NVLink as they leave
the tensor cores (torch_mcpu_b200.symm.mm_allreduce).
"""

from __future__ import annotations

import torch

from . import ops


class TPShardSwiGLU:
    """One rank's shard.  w_gate_up: [2*I_r, H] as [gate_r; up_r] (nn.Linear
    layout), w_down: [H, I_r], rms_weight: [H] or None.  All bf16."""

    def __init__(self, w_gate_up: torch.Tensor, w_down: torch.Tensor,
                 rms_weight: torch.Tensor | None = None, eps: float = 1e-6):
        if w_gate_up.dtype != torch.bfloat16 or w_down.dtype != torch.bfloat16:
            raise RuntimeError("TPShardSwiGLU: bfloat16 weights expected")
        self.I = w_gate_up.shape[0] // 2
        self.H = w_gate_up.shape[1]
        if tuple(w_down.shape) != (self.H, self.I):
            raise RuntimeError(f"TPShardSwiGLU: w_down must be [{self.H}, {self.I}]")
        self.w_gu = ops.interleave_gate_up(w_gate_up.contiguous())
        self.w_down = w_down.contiguous()
        self.rms_weight = None if rms_weight is None else rms_weight.contiguous()
        self.eps = eps
        self._bufs: dict = {}

    def _buf(self, name: str, shape, device) -> torch.Tensor:
        t = self._bufs.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.device != device:
            t = torch.empty(shape, dtype=torch.bfloat16, device=device)
            self._bufs[name] = t
        return t

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Partial output y_r [T, H] of this rank (before the all-reduce)."""
        T = x.shape[0]
        h = x
        if self.rms_weight is not None:
            h = self._buf("normed", (T, self.H), x.device)
            ops.rms_norm(h, x, self.rms_weight, self.eps)
        a = self._buf("act", (T, self.I), x.device)
        ops.gemm_swiglu(h, self.w_gu, out=a)
        if out is None:
            out = torch.empty(T, self.H, dtype=torch.bfloat16, device=x.device)
        return ops.mm_nt(a, self.w_down, out=out)

    __call__ = forward

    def flops(self, tokens: int) -> int:
        return 2 * tokens * self.H * self.I * 3


def run_one_step(model: TPShardSwiGLU, x: torch.Tensor, group=None, out=None) -> torch.Tensor:
    """forward + SUM all-reduce over the tensor-parallel group
    (example/01_mlp_tp4/run.py:106-113)."""
    y = model(x, out=out)
    if group is not None or (torch.distributed.is_available() and torch.distributed.is_initialized()):
        if torch.distributed.get_world_size(group) > 1:
            torch.distributed.all_reduce(y, group=group)
    return y


def mcpu_tp_step(x: torch.Tensor, w_gate_up_interleaved: torch.Tensor, w_down: torch.Tensor,
                 act: torch.Tensor, window=None, out: torch.Tensor | None = None, group=None) -> torch.Tensor:
    """One TP MLP step on mcpu tensors (example/01_mlp_tp4/run.py:106-113):
    fused gate/up GEMM + SwiGLU into `act` [T, I_r], then the row-parallel
    down projection and the SUM all-reduce, either fused over the symmetric
    `window` (the result is a view of the window) or as mm into `out` plus
    an all_reduce through the mcpu ProcessGroup (NCCL)."""
    torch.ops.mcpu.gemm_swiglu.out(x, w_gate_up_interleaved, out=act)
    if window is not None:
        from .symm import mm_allreduce

        return mm_allreduce(act, w_down, window)
    if out is None:
        out = torch.empty(x.shape[0], w_down.shape[0], dtype=torch.bfloat16, device=x.device)
    torch.mm(act, w_down.t(), out=out)
    if torch.distributed.is_available() and torch.distributed.is_initialized():
        if torch.distributed.get_world_size(group) > 1:
            torch.distributed.all_reduce(out, group=group)
    return out
