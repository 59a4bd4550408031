"""torch_mcpu on B200: the mcpu device hot path as sm_100a CUDA.

The product is the C-ABI library libtorch_mcpu_b200.so (include/openreg.h,
include/mcpu_ops.h); this package builds it in-tree and exposes the ops with
the reference's Python signatures.
"""

from . import _lib  # noqa: F401
from .ops import grouped_topk, grouped_topk_exact_rows, rms_norm, silu_and_mul  # noqa: F401

__all__ = ["grouped_topk", "grouped_topk_exact_rows", "silu_and_mul", "rms_norm"]
