"""Builds the PyTorch-facing extension of the mcpu device in-tree.

    python -m torch_mcpu_b200.build_ext   # -> torch_mcpu_b200/_ext_build/torch_mcpu_b200_C.so

The extension (csrc_torch/*.cpp: PrivateUse1 allocator, guard, hooks, aten
and mcpu:: registrations, the NCCL ProcessGroup, the Python methods) is a
host-only layer over libtorch_mcpu_b200.so; it links that library with a
relative rpath and NCCL from the PyTorch wheel.
"""

from __future__ import annotations

import glob
import os
import sys

from . import build as _cabi

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc_torch")
OUT = os.path.join(HERE, "_ext_build")
NAME = "torch_mcpu_b200_C"
SO = os.path.join(OUT, NAME + ".so")


def _nccl_dirs():
    import nvidia.nccl as nccl  # the NCCL PyTorch itself loads

    base = os.path.dirname(nccl.__file__) if getattr(nccl, "__file__", None) else list(nccl.__path__)[0]
    return os.path.join(base, "include"), os.path.join(base, "lib")


def sources():
    return sorted(glob.glob(os.path.join(SRC, "*.cpp")))


def up_to_date() -> bool:
    if not os.path.exists(SO):
        return False
    deps = sources() + glob.glob(os.path.join(SRC, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return os.path.getmtime(SO) >= max(os.path.getmtime(f) for f in deps)


def _use_shared_libstdcxx_compiler() -> None:
    """The extension has to share libstdc++ with torch: a private static copy
    (what a toolchain gives when its shared libstdc++ cannot be found) has its
    own iostream and locale objects, and torch's error messages, formatted
    with torch's streams, then crash when they print a number.  The system
    g++ links libstdc++ dynamically, so it builds the extension when present."""
    for cxx, cc in (("/usr/bin/g++", "/usr/bin/gcc"),):
        if os.path.exists(cxx):
            os.environ["CXX"] = cxx
            if os.path.exists(cc):
                os.environ["CC"] = cc
            return


def build(verbose: bool = False) -> str:
    _cabi.build()
    if up_to_date():
        return SO
    _use_shared_libstdcxx_compiler()
    from torch.utils import cpp_extension

    nccl_inc, nccl_lib = _nccl_dirs()
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    os.makedirs(OUT, exist_ok=True)
    cpp_extension.load(
        name=NAME,
        sources=sources(),
        build_directory=OUT,
        extra_include_paths=[os.path.join(ROOT, "include"), SRC, nccl_inc, cuda_inc],
        extra_cflags=["-O2", "-std=c++17", "-fvisibility=hidden"],
        extra_ldflags=[
            f"-L{HERE}", "-ltorch_mcpu_b200", "-Wl,-rpath,'$$ORIGIN/..'",
            f"-L{nccl_lib}", "-l:libnccl.so.2", f"-Wl,-rpath,{nccl_lib}",
        ],
        with_cuda=False,
        is_python_module=True,
        verbose=verbose,
    )
    return SO


CHECK_SRC = os.path.join(ROOT, "tests", "launch_api", "launch_check.cu")
CHECK_NAME = "mcpu_launch_check"
CHECK_SO = os.path.join(OUT, CHECK_NAME + ".so")


def build_launch_check(verbose: bool = False) -> str:
    """The launch-API caller used by tests/test_launch_api_gpu.py: compiled
    by nvcc for sm_100a against include/mcpu_launch.h, linked to the
    extension that exports the API's functions."""
    build()
    deps = [CHECK_SRC, SO, os.path.join(ROOT, "include", "mcpu_launch.h")]
    if os.path.exists(CHECK_SO) and os.path.getmtime(CHECK_SO) >= max(os.path.getmtime(f) for f in deps):
        return CHECK_SO
    _use_shared_libstdcxx_compiler()
    from torch.utils import cpp_extension

    cpp_extension.load(
        name=CHECK_NAME,
        sources=[CHECK_SRC],
        build_directory=OUT,
        extra_include_paths=[os.path.join(ROOT, "include")],
        extra_cflags=["-O2", "-std=c++17"],
        extra_cuda_cflags=["-O2", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a"],
        extra_ldflags=[f"-L{OUT}", f"-l:{NAME}.so", "-Wl,-rpath,'$$ORIGIN'"],
        with_cuda=True,
        is_python_module=True,
        verbose=verbose,
    )
    return CHECK_SO


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    if "--launch-check" in sys.argv:
        print(build_launch_check(verbose="-v" in sys.argv))
