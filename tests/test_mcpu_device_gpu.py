"""The PyTorch "mcpu" device on B200: tensors, copies, the hot aten ops and
the mcpu:: custom ops, as the reference's users drive them
(tests/test_ops.py, test_streams.py, test_memory.py of kzwrime/torch_mcpu in
spirit; results checked against the oracle or a PyTorch fp32 reference)."""

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mcpu():
    import torch_mcpu_b200.device as d

    assert torch.mcpu.is_available()
    return d


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_tensor_round_trip_and_dtype_conversion(mcpu):
    x = torch.randn(5, 7)
    y = x.to("mcpu")
    assert y.device.type == "mcpu" and y.is_mcpu
    assert torch.equal(y.cpu(), x)
    assert torch.equal(y.to(torch.bfloat16).cpu(), x.to(torch.bfloat16))
    assert torch.equal(y.t().contiguous().cpu(), x.t().contiguous())
    assert torch.equal(y[1:4, ::2].cpu(), x[1:4, ::2])
    assert torch.equal(y.to(torch.int32).cpu(), x.to(torch.int32))
    assert y[2, 3].item() == x[2, 3].item()


def test_fill_zero_empty_resize(mcpu):
    y = torch.empty(3, 4, device="mcpu")
    y.fill_(2.5)
    assert torch.equal(y.cpu(), torch.full((3, 4), 2.5))
    y.zero_()
    assert torch.equal(y.cpu(), torch.zeros(3, 4))
    z = torch.zeros(4, 6, dtype=torch.bfloat16, device="mcpu")
    z[:, 1::2].fill_(1.0)
    ref = torch.zeros(4, 6, dtype=torch.bfloat16)
    ref[:, 1::2] = 1.0
    assert torch.equal(z.cpu(), ref)
    w = torch.empty(2, device="mcpu")
    w.resize_(100)
    assert w.numel() == 100


def test_mm_addmm_on_mcpu_tensors(mcpu):
    g = torch.Generator().manual_seed(0)
    a = torch.randn(300, 512, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(640, 512, generator=g)).to(torch.bfloat16)
    bias = torch.randn(640, generator=g).to(torch.bfloat16)
    out = torch.mm(a.to("mcpu"), w.to("mcpu").t()).cpu().float()
    ref = a.float() @ w.float().t()
    assert (out - ref).norm() / ref.norm() < 5e-3
    out2 = torch.addmm(bias.to("mcpu"), a.to("mcpu"), w.to("mcpu").t()).cpu().float()
    ref2 = ref + bias.float()
    assert (out2 - ref2).norm() / ref2.norm() < 5e-3
    # the example's structure: mm(x, w.t()) + b would need aten::add; addmm covers it


def test_sigmoid_silu_mul_match_the_raw_loops(mcpu):
    x = torch.linspace(-20, 20, 4001)
    s = torch.sigmoid(x.to("mcpu")).cpu()
    np.testing.assert_array_equal(s.numpy(), oracle.sigmoid_f32(x.numpy(), oracle.EXP_CR))
    xb = C.silu_inputs(32, 256)
    gate, up = xb[:, :256].contiguous(), xb[:, 256:].contiguous()
    act = torch.nn.functional.silu(gate.to("mcpu"))
    prod = (act * up.to("mcpu")).cpu()
    np.testing.assert_array_equal(bits(prod), oracle.silu_and_mul_bf16(bits(xb), exp_mode=oracle.EXP_CR))


def test_custom_ops_on_mcpu_tensors(mcpu):
    cfg = C.deepseek_v3(1024)
    gating, bias = C.router_inputs(cfg)
    w, ids = torch.ops.mcpu.grouped_topk(gating.to("mcpu"), 8, 4, 8, True, 2.5, bias.to("mcpu"), "sigmoid")
    ow, oids, _, _ = oracle.grouped_topk(gating.numpy(), 8, True, 8, 4, "sigmoid", 2.5, bias.numpy(),
                                         exp_mode=oracle.EXP_CR)
    np.testing.assert_array_equal(np.sort(ids.cpu().numpy(), 1), np.sort(oids, 1))
    x = C.silu_inputs(16, 1024)
    out = torch.empty(16, 1024, dtype=torch.bfloat16, device="mcpu")
    torch.ops.mcpu.silu_and_mul(out, x.to("mcpu"))
    np.testing.assert_array_equal(bits(out.cpu()), oracle.silu_and_mul_bf16(bits(x), exp_mode=oracle.EXP_CR))
    xr, wr = C.rms_inputs(8, 7168)
    o = torch.empty(8, 7168, dtype=torch.bfloat16, device="mcpu")
    torch.ops.mcpu.rms_norm(o, xr.to("mcpu"), wr.to("mcpu"), 1e-6)
    np.testing.assert_array_equal(bits(o.cpu()), oracle.rms_norm_bf16(bits(xr), bits(wr), 1e-6))


def test_unregistered_op_raises_no_cpu_fallback(mcpu):
    y = torch.ones(4, device="mcpu")
    with pytest.raises(NotImplementedError):
        torch.cumsum(y, 0)


def test_streams_events_and_record_stream(mcpu):
    s = torch.Stream(device="mcpu")
    e0 = torch.Event(device="mcpu", enable_timing=True)
    e1 = torch.Event(device="mcpu", enable_timing=True)
    x = torch.randn(1024, 1024).to(torch.bfloat16).to("mcpu")
    e0.record(s)
    torch.mcpu.synchronize()
    e1.record(s)
    e1.synchronize()
    assert e0.elapsed_time(e1) >= 0.0
    x.record_stream(s)
    del x
    torch.mcpu.synchronize()


def test_memory_stats_track_allocations(mcpu):
    torch.mcpu.synchronize()
    base = torch.mcpu.memory_allocated()
    t = torch.empty(1 << 20, dtype=torch.float32, device="mcpu")
    assert torch.mcpu.memory_allocated() - base == 4 << 20
    assert torch.mcpu.max_memory_allocated() >= base + (4 << 20)
    del t
    assert torch.mcpu.memory_allocated() == base
    torch.mcpu.empty_cache()


def test_device_module_api(mcpu):
    free, total = torch.mcpu.mem_get_info()
    assert 0 < free <= total
    with torch.mcpu.device(0):
        assert torch.mcpu.current_device() == 0
    t = torch.empty(1 << 20, device="mcpu")
    assert torch.mcpu.memory_reserved() >= 4 << 20
    assert torch.mcpu.max_memory_reserved() >= torch.mcpu.memory_reserved()
    del t
    d = torch.mcpu.default_stream()
    assert d.device_type == torch.device("mcpu").type or d.device.type == "mcpu"


def test_graph_capture_and_replay(mcpu):
    g = torch.Generator().manual_seed(5)
    a = torch.randn(256, 512, generator=g).to(torch.bfloat16).to("mcpu")
    w = (0.05 * torch.randn(384, 512, generator=g)).to(torch.bfloat16).to("mcpu")
    out = torch.empty(256, 384, dtype=torch.bfloat16, device="mcpu")
    side = torch.mcpu.Stream()
    graph = torch.mcpu.Graph()
    with torch.mcpu.stream(side):
        torch.mm(a, w.t(), out=out)  # first call configures the kernel outside the capture
        side.synchronize()
        ref = out.cpu().clone()
        out.zero_()
        with graph.capture():
            torch.mm(a, w.t(), out=out)
        side.synchronize()
        assert torch.equal(out.cpu(), torch.zeros(256, 384, dtype=torch.bfloat16))  # captured, not run
        graph.replay()
        side.synchronize()
    assert torch.equal(out.cpu(), ref)
    graph.reset()
