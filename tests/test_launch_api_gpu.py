"""The kernel-launch API (include/mcpu_launch.h) from a caller compiled
against it (tests/launch_api/launch_check.cu): host callables run in stream
order around device work, MCPU_LAUNCH_TIMED_KERNEL records timing events,
the tensor-selected stream is the tensor's current mcpu stream, and the
__global__ overload launches device kernels — the uses of McpuKernelLaunch.h
in kzwrime/torch_mcpu's op files (e.g. csrc/aten/ops/cumsum.cpp:29)."""

import importlib.util
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lc():
    import torch_mcpu_b200.device  # noqa: F401  (loads the extension the module links to)
    from torch_mcpu_b200 import build_ext

    path = build_ext.CHECK_SO
    if not os.path.exists(path):
        path = build_ext.build_launch_check()
    spec = importlib.util.spec_from_file_location(build_ext.CHECK_NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_host_tasks_run_in_stream_order_around_device_work(lc):
    t = torch.zeros(1000, device="mcpu")
    lc.timing(True, True)
    assert lc.host_tasks(t) == [1, 2, 3, 4]
    ref = 10.0 + torch.arange(1000, dtype=torch.float32)
    assert torch.equal(t.cpu(), ref)
    n, *span = lc.timing(False, False)
    assert n == 1 and span[0] >= 0.0


def test_global_kernel_overload_and_timed_launch(lc):
    t = torch.empty(4097, device="mcpu")
    lc.device_fill(t, 1.5, False)
    assert torch.equal(t.cpu(), 1.5 + torch.arange(4097, dtype=torch.float32))
    lc.timing(True, True)
    lc.device_fill(t, -2.0, True)
    lc.device_fill(t, 3.0, True)
    torch.mcpu.synchronize()
    n, span = lc.timing(False, False)
    assert n == 2 and span > 0.0
    assert torch.equal(t.cpu(), 3.0 + torch.arange(4097, dtype=torch.float32))


def test_launch_on_a_side_stream_follows_that_stream(lc):
    s = torch.mcpu.Stream()
    t = torch.zeros(256, device="mcpu")
    torch.mcpu.synchronize()
    with torch.mcpu.stream(s):
        assert torch.mcpu.current_stream() == s
        lc.device_fill(t, 7.0, False)
    assert torch.mcpu.current_stream() == torch.mcpu.default_stream()
    s.synchronize()
    assert torch.equal(t.cpu(), 7.0 + torch.arange(256, dtype=torch.float32))


def test_kernel_timing_module_api(lc):
    torch.mcpu.set_kernel_timing_enabled(True)
    torch.mcpu.reset_kernel_timing()
    t = torch.empty(64, device="mcpu")
    lc.device_fill(t, 0.0, True)
    torch.mcpu.synchronize()
    snap = torch.mcpu.get_kernel_timing()
    torch.mcpu.set_kernel_timing_enabled(False)
    ev = snap[0]["events"]
    assert len(ev) == 1 and ev[0]["name"] == "launch_check.fill" and ev[0]["elapsed_time"] >= 0.0
