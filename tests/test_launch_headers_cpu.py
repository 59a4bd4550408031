"""The launch API through the reference's header paths, for out-of-tree op
files written against kzwrime/torch_mcpu: they include
<runtime/McpuKernelLaunch.h> (example/02_external_mcpu_kernel_demo/
external_axpby.cpp:6 there) with `torch_mcpu.get_include()` on the include
path.  Compile checks with the host compiler (no GPU, no linking):

* tests/launch_api/runtime_headers_check.cpp instantiates every launch form
  (tensor-selected stream, named and timed launches, move-only payloads,
  MCPU_LAUNCH_TIMED_KERNEL, orLaunchKernel, the memory guards, the timing
  log);
* the reference's own external_axpby.cpp, unchanged, when a checkout of the
  reference is named by TORCH_MCPU_REFERENCE (skipped otherwise).  It
  compiles as it is; at run time its host lambda dereferences device
  pointers, which the B200 launch API does not allow (a host callable must
  launch a __global__ function through the launch_kernel overload instead).
"""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _syntax_check(src):
    from torch.utils import cpp_extension

    import torch_mcpu

    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no host C++ compiler")
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    cmd = [cxx, "-std=c++17", "-fsyntax-only", "-D_GLIBCXX_USE_CXX11_ABI=1", f"-I{torch_mcpu.get_include()}",
           f"-I{cuda_inc}"]
    cmd += [f"-I{p}" for p in cpp_extension.include_paths()]
    cmd.append(src)
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]


def test_every_launch_form_compiles_through_the_reference_header_paths():
    _syntax_check(os.path.join(ROOT, "tests", "launch_api", "runtime_headers_check.cpp"))


def test_reference_external_op_example_compiles_unchanged():
    ref = os.environ.get("TORCH_MCPU_REFERENCE")
    if not ref:
        pytest.skip("TORCH_MCPU_REFERENCE does not name a checkout of the reference")
    src = os.path.join(ref, "example", "02_external_mcpu_kernel_demo", "external_axpby.cpp")
    if not os.path.exists(src):
        pytest.skip(f"{src} not found")
    _syntax_check(src)


def test_torch_mcpu_import_name_and_extension_helpers():
    import torch

    import torch_mcpu

    assert hasattr(torch, "mcpu") and torch_mcpu.openreg.device_count() >= 0
    assert os.path.exists(os.path.join(torch_mcpu.get_include(), "runtime", "McpuKernelLaunch.h"))
    assert torch_mcpu.get_compile_definitions()["TORCH_MCPU_ENABLE_SYNC_KERNEL_LAUNCH"] == "0"
    assert "-DTORCH_MCPU_ENABLE_CPU_FALLBACK=0" in torch_mcpu.get_compile_flags()


def test_reference_schema_block_is_registered():
    """The six schemas of the reference's TORCH_LIBRARY(mcpu) block
    (csrc/aten/OpenRegExtra.cpp:147-162), unchanged."""
    import torch

    import torch_mcpu  # noqa: F401

    want = {
        "custom_abs": "mcpu::custom_abs(Tensor input) -> Tensor",
        "stream_sleep_fill_": "mcpu::stream_sleep_fill_(Tensor(a!) input, int value, int sleep_ms) -> Tensor(a!)",
        "stream_sleep_copy_": "mcpu::stream_sleep_copy_(Tensor(a!) dst, Tensor src, int sleep_ms) -> Tensor(a!)",
        "first_element_int": "mcpu::first_element_int(Tensor input) -> int",
        "kernel_launch_lifetime_counts":
            "mcpu::kernel_launch_lifetime_counts(Tensor stream_selector, int launches) -> (int, int, int)",
        "kernel_launch_failed_lifetime_counts":
            "mcpu::kernel_launch_failed_lifetime_counts(Tensor stream_selector) -> (int, int, int)",
    }
    for name, schema in want.items():
        assert str(getattr(torch.ops.mcpu, name).default._schema) == schema
