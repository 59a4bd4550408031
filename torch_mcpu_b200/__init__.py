"""torch_mcpu on B200: the mcpu device hot path as sm_100a CUDA.

The product is the C-ABI library libtorch_mcpu_b200.so (include/openreg.h,
include/mcpu_ops.h); this package builds it in-tree and exposes the ops with
the reference's Python signatures.
"""

from . import _lib  # noqa: F401
from .ops import (  # noqa: F401
    device_error,
    gemm_swiglu,
    grouped_topk,
    grouped_topk_exact_rows,
    grouped_topk_moe_align,
    interleave_gate_up,
    mm_nt,
    rms_norm,
    sigmoid,
    silu,
    silu_and_mul,
)

__all__ = ["grouped_topk", "grouped_topk_exact_rows", "grouped_topk_moe_align", "silu_and_mul", "rms_norm", "mm_nt",
           "gemm_swiglu", "interleave_gate_up", "device_error", "sigmoid", "silu"]
