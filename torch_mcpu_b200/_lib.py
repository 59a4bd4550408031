"""ctypes view of libtorch_mcpu_b200.so (the C-ABI in include/*.h).

The library is built in-tree (torch_mcpu_b200/build.py).  Loading fails
loudly when it is missing: there is no CPU fallback for any op.
"""

from __future__ import annotations

import ctypes
import os

from . import build as _build

_lib = None

c_int, c_int64, c_float, c_void_p = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p

SYMM_MAX_RANKS = 8
SYMM_HANDLE_BYTES = 64


class SymmWindow(ctypes.Structure):
    """mcpuSymmWindow of include/mcpu_ops.h."""

    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("bytes", ctypes.c_uint64),
                ("base", c_void_p * SYMM_MAX_RANKS)]


# name -> (restype, argtypes); every entry point declared in include/*.h
SIGNATURES = {
    # include/openreg.h
    "orMalloc": (c_int, [ctypes.POINTER(c_void_p), ctypes.c_size_t]),
    "orFree": (c_int, [c_void_p]),
    "orMallocHost": (c_int, [ctypes.POINTER(c_void_p), ctypes.c_size_t]),
    "orFreeHost": (c_int, [c_void_p]),
    "orMemcpy": (c_int, [c_void_p, c_void_p, ctypes.c_size_t, c_int]),
    "orMemcpyAsync": (c_int, [c_void_p, c_void_p, ctypes.c_size_t, c_int, c_void_p]),
    "orPointerGetAttributes": (c_int, [c_void_p, c_void_p]),
    "orMemoryUnprotect": (c_int, [c_void_p]),
    "orMallocAsync": (c_int, [ctypes.POINTER(c_void_p), ctypes.c_size_t, c_void_p]),
    "orFreeAsync": (c_int, [c_void_p, c_void_p]),
    "orMemPoolTrim": (c_int, [ctypes.c_size_t]),
    "orMemoryProtect": (c_int, [c_void_p]),
    "orGetDeviceCount": (c_int, [ctypes.POINTER(c_int)]),
    "orSetDevice": (c_int, [c_int]),
    "orGetDevice": (c_int, [ctypes.POINTER(c_int)]),
    "orDeviceGetStreamPriorityRange": (c_int, [ctypes.POINTER(c_int), ctypes.POINTER(c_int)]),
    "orDeviceSynchronize": (c_int, []),
    "orStreamCreateWithPriority": (c_int, [ctypes.POINTER(c_void_p), ctypes.c_uint, c_int]),
    "orStreamCreate": (c_int, [ctypes.POINTER(c_void_p)]),
    "orStreamGetPriority": (c_int, [c_void_p, ctypes.POINTER(c_int)]),
    "orStreamDestroy": (c_int, [c_void_p]),
    "orStreamQuery": (c_int, [c_void_p]),
    "orStreamSynchronize": (c_int, [c_void_p]),
    "orStreamWaitEvent": (c_int, [c_void_p, c_void_p, ctypes.c_uint]),
    "orEventCreateWithFlags": (c_int, [ctypes.POINTER(c_void_p), ctypes.c_uint]),
    "orEventCreate": (c_int, [ctypes.POINTER(c_void_p)]),
    "orEventDestroy": (c_int, [c_void_p]),
    "orEventRecord": (c_int, [c_void_p, c_void_p]),
    "orEventSynchronize": (c_int, [c_void_p]),
    "orEventQuery": (c_int, [c_void_p]),
    "orEventElapsedTime": (c_int, [ctypes.POINTER(c_float), c_void_p, c_void_p]),
    # include/mcpu_ops.h
    "mcpuGetLastErrorString": (ctypes.c_char_p, []),
    "mcpu_grouped_topk": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_int,
                                  c_float, c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "mcpu_grouped_topk_exact_rows": (c_int, [ctypes.POINTER(ctypes.c_ulonglong), c_int]),
    "mcpu_grouped_topk_moe_align": (c_int, [c_void_p, c_int, c_int64, c_int, c_int, c_int, c_int, c_int, c_float,
                                            c_void_p, c_int, c_void_p, c_void_p, c_int, c_void_p, c_int64, c_void_p,
                                            c_int64, c_void_p, c_void_p, ctypes.c_uint64, c_void_p]),
    "mcpu_grouped_topk_moe_align_workspace_bytes": (c_int, [c_int64, c_int, c_int, ctypes.POINTER(ctypes.c_uint64)]),
    "mcpu_silu_and_mul": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int, c_void_p]),
    "mcpu_rms_norm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_float, c_int, c_void_p]),
    "mcpu_mm": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p]),
    "mcpu_addmm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                           c_void_p]),
    "mcpu_gemm_swiglu": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                                 c_void_p]),
    "mcpu_symm_alloc": (c_int, [ctypes.c_uint64, ctypes.POINTER(c_void_p), c_void_p]),
    "mcpu_symm_open": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "mcpu_symm_close": (c_int, [c_void_p]),
    "mcpu_symm_free": (c_int, [c_void_p]),
    "mcpu_symm_clear": (c_int, [c_void_p, ctypes.c_uint64, c_void_p]),
    "mcpu_mm_allreduce": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int,
                                  ctypes.POINTER(SymmWindow), ctypes.POINTER(c_void_p), c_void_p]),
    "mcpu_mm_allreduce_window_bytes": (c_int, [c_int64, c_int64, c_int, ctypes.POINTER(ctypes.c_uint64)]),
    "mcpu_mm_allreduce_control_bytes": (c_int, [ctypes.c_uint64, c_int, ctypes.POINTER(ctypes.c_uint64)]),
    "mcpu_moe_align_block_size": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_int64, c_void_p, c_int64,
                                          c_void_p, c_void_p, ctypes.c_uint64, c_void_p]),
    "mcpu_moe_align_workspace_bytes": (c_int, [c_int64, c_int, ctypes.POINTER(ctypes.c_uint64)]),
    "mcpu_moe_align_block_size_static": (c_int, [c_void_p, c_int64, c_int, c_int, c_void_p, c_int64, c_void_p,
                                                 c_int64, c_void_p, c_void_p]),
    "mcpu_stream_sleep_fill_i64": (c_int, [c_void_p, c_int64, c_int64, c_int64, c_void_p]),
    "mcpu_stream_sleep_copy_i64": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "mcpu_read_i64_now": (c_int, [c_void_p, c_void_p]),
    "mcpu_vllm_min_p": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p]),
    "mcpu_vllm_topk_log_softmax": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_int64, c_int64,
                                           c_int64, c_void_p]),
    "mcpu_vllm_ranks": (c_int, [c_void_p, c_void_p, c_int, c_int64, c_int64, c_void_p, c_int64, c_void_p]),
    "mcpu_vllm_penalties": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                    c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_void_p, c_int64, c_int64,
                                    c_int64, c_void_p]),
    "mcpu_vllm_bias": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p, c_void_p,
                               c_int64, c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_int64, c_int64, c_void_p,
                               c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "mcpu_vllm_bad_words": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                                    c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                    c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mcpu_vllm_bincount": (c_int, [c_void_p, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_int64,
                                   c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p]),
    "mcpu_device_error": (c_int, [ctypes.POINTER(c_int), c_int]),
    "mcpu_mem_get_info": (c_int, [c_int, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
    "mcpu_mem_pool_reserved": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "mcpu_graph_capture_begin": (c_int, [c_void_p]),
    "mcpu_graph_capture_end": (c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    "mcpu_graph_launch": (c_int, [c_void_p, c_void_p]),
    "mcpu_graph_destroy": (c_int, [c_void_p]),
    "mcpu_binary": (c_int, [c_int, c_void_p, c_int, ctypes.POINTER(ctypes.c_int64), c_void_p, c_int, ctypes.POINTER(ctypes.c_int64), c_void_p, c_int, ctypes.POINTER(ctypes.c_int64), c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_double, c_void_p]),
    "mcpu_unary": (c_int, [c_int, c_void_p, c_int, ctypes.POINTER(ctypes.c_int64), c_void_p, c_int, ctypes.POINTER(ctypes.c_int64), c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_double, c_void_p]),
    "mcpu_masked_fill": (c_int, [c_void_p, c_int, ctypes.POINTER(ctypes.c_int64), c_void_p, ctypes.POINTER(ctypes.c_int64), c_int, ctypes.POINTER(ctypes.c_int64), ctypes.c_double, ctypes.c_int64, c_int, c_void_p]),
    "mcpu_reduce_lastdim": (c_int, [c_int, c_void_p, c_int, ctypes.c_int64, ctypes.c_int64, c_void_p, c_int, c_void_p, c_void_p]),
    "mcpu_topk_lastdim": (c_int, [c_void_p, c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, c_int, c_void_p, c_void_p, c_void_p]),
    "mcpu_softmax_lastdim": (c_int, [c_void_p, c_int, ctypes.c_int64, ctypes.c_int64, c_void_p, c_int, c_int, c_void_p]),
    "mcpu_gather": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), ctypes.c_int64, c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), c_void_p, ctypes.POINTER(ctypes.c_int64), c_void_p]),
    "mcpu_scatter_value": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), ctypes.c_int64, c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64), ctypes.c_double, ctypes.c_int64, c_int, c_void_p]),
    "mcpu_copy_strided": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                  c_void_p]),
    "mcpu_fill": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, ctypes.c_double, c_int64, c_int,
                          c_void_p]),
    "mcpu_sigmoid": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "mcpu_silu": (c_int, [c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "mcpu_mul": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
}


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True):
    """Load the device library, building it first when it is missing (or,
    with MCPU_AUTOBUILD=1, older than its sources)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    stale = os.environ.get("MCPU_AUTOBUILD") == "1" and not _build.up_to_date()
    if build_if_missing and (not os.path.exists(path) or stale):
        _build.build()
    if not os.path.exists(path):
        raise RuntimeError(f"mcpu device library not built: {path} is missing "
                           "(run python -m torch_mcpu_b200.build)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


ERROR_NAMES = {0: "orSuccess", 1: "orErrorUnknown", 2: "orErrorNotReady", 3: "orErrorTimeout",
               4: "orErrorInvalidValue"}


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().mcpuGetLastErrorString().decode(errors="replace")
        raise RuntimeError(f"{what} failed ({ERROR_NAMES.get(rc, rc)}): {msg}")
