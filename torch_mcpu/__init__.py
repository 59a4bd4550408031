"""`import torch_mcpu` for code written against kzwrime/torch_mcpu.

The reference's package (torch_mcpu/__init__.py:13-39 there) registers its
CPU-simulated device; this one registers the same "mcpu" device backed by
the B200 (torch_mcpu_b200.device): the PrivateUse1 backend renamed to
"mcpu", the torch.mcpu module, the tensor methods and the "mcpu"
distributed backend (NCCL).  It also provides the helpers out-of-tree op
libraries call (torch_mcpu/paths.py, compile_flags.py there):

    get_include()             directory holding runtime/McpuKernelLaunch.h
    get_library_dir()         directory of the library exporting the launch
                              API (torch_mcpu_b200_C.so)
    get_compile_definitions() / get_compile_flags() / get_compile_config()
"""

from __future__ import annotations

import os

import torch_mcpu_b200.device as openreg  # noqa: F401  (registers the device)
from torch_mcpu_b200 import build_ext as _build_ext

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# The reference records its CMake options for extensions to mirror.  On
# B200 kernels are enqueued on CUDA streams (never run synchronously at
# launch) and there is no CPU fallback.
_COMPILE_DEFINITIONS = {
    "TORCH_MCPU_ENABLE_SYNC_KERNEL_LAUNCH": "0",
    "TORCH_MCPU_ENABLE_CPU_FALLBACK": "0",
}


def get_include() -> str:
    """Directory external C++ extensions add to their include path."""
    return os.path.join(_ROOT, "include")


def get_library_dir() -> str:
    """Directory of torch_mcpu_b200_C.so, which exports the launch API."""
    return os.path.dirname(_build_ext.SO)


def get_compile_config() -> dict:
    return {"definitions": dict(_COMPILE_DEFINITIONS),
            "compile_flags": [f"-D{k}={v}" for k, v in _COMPILE_DEFINITIONS.items()]}


def get_compile_definitions() -> dict:
    return dict(_COMPILE_DEFINITIONS)


def get_compile_flags() -> list:
    return list(get_compile_config()["compile_flags"])
