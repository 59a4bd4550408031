"""The reference's own TORCH_LIBRARY(mcpu) ops on the B200 mcpu device
(schemas csrc/aten/OpenRegExtra.cpp:147-162, bodies csrc/aten/native/
Extra.cpp:251-353 of kzwrime/torch_mcpu), used the way its tests use them
(tests/test_streams.py:150-230): a fill or copy that waits on its stream
is not visible before the stream is synchronised, device synchronisation
and stream-on-stream waits order it, first_element_int reads at once, and
the launch API's move-only payloads are constructed, run and destroyed
once each (or never run when the launch is refused)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mcpu():
    import torch_mcpu  # noqa: F401  (the reference's import name)

    assert torch.mcpu.is_available()
    return torch


def _t(v, n=16):
    return torch.full((n,), v, dtype=torch.int64).to("mcpu")


def test_stream_async_native_op(mcpu):
    s = torch.mcpu.Stream()
    x = _t(0)
    torch.mcpu.synchronize()
    with torch.mcpu.stream(s):
        torch.ops.mcpu.stream_sleep_fill_(x, 7, 300)
    if not s.query():
        assert torch.ops.mcpu.first_element_int(x) == 0
    s.synchronize()
    assert s.query()
    assert torch.ops.mcpu.first_element_int(x) == 7
    assert torch.equal(x.cpu(), torch.full((16,), 7, dtype=torch.int64))


def test_device_synchronize_waits_for_stream_native_op(mcpu):
    s = torch.mcpu.Stream()
    x = _t(0)
    torch.mcpu.synchronize()
    with torch.mcpu.stream(s):
        torch.ops.mcpu.stream_sleep_fill_(x, 13, 300)
    assert torch.ops.mcpu.first_element_int(x) == 0
    torch.mcpu.synchronize()
    assert s.query()
    assert torch.ops.mcpu.first_element_int(x) == 13


def test_stream_wait_stream_orders_native_ops(mcpu):
    producer, consumer = torch.mcpu.Stream(), torch.mcpu.Stream()
    src, dst = _t(0, 1000), _t(-1, 1000)
    torch.mcpu.synchronize()
    with torch.mcpu.stream(producer):
        torch.ops.mcpu.stream_sleep_fill_(src, 11, 500)
    with torch.mcpu.stream(consumer):
        consumer.wait_stream(producer)
        torch.ops.mcpu.stream_sleep_copy_(dst, src, 0)
    assert torch.ops.mcpu.first_element_int(dst) == -1
    consumer.synchronize()
    assert torch.ops.mcpu.first_element_int(dst) == 11
    assert torch.ops.mcpu.first_element_int(src) == 11
    assert torch.equal(dst.cpu(), torch.full((1000,), 11, dtype=torch.int64))


def test_stream_test_ops_reject_what_the_reference_rejects(mcpu):
    with pytest.raises(RuntimeError, match="int64"):
        torch.ops.mcpu.stream_sleep_fill_(torch.zeros(4).to("mcpu"), 1, 0)
    with pytest.raises(RuntimeError, match="identical shapes"):
        torch.ops.mcpu.stream_sleep_copy_(_t(0, 4), _t(0, 5), 0)
    with pytest.raises(RuntimeError, match="non-empty"):
        torch.ops.mcpu.first_element_int(torch.zeros(0, dtype=torch.int64).to("mcpu"))


def test_kernel_launch_lifetime_counts(mcpu):
    assert tuple(torch.ops.mcpu.kernel_launch_lifetime_counts(_t(0), 6)) == (6, 6, 6)
    assert tuple(torch.ops.mcpu.kernel_launch_lifetime_counts(_t(0), 0)) == (0, 0, 0)


def test_kernel_launch_failed_lifetime_counts(mcpu):
    assert tuple(torch.ops.mcpu.kernel_launch_failed_lifetime_counts(_t(0))) == (1, 1, 0)


def test_custom_abs(mcpu):
    x = torch.tensor([-1.5, 2.0, -0.0, -3.25])
    assert torch.equal(torch.ops.mcpu.custom_abs(x.to("mcpu")).cpu(), x.abs())
