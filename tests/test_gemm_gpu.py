"""tcgen05 bf16 GEMM (mm, addmm, fused gate/up + silu_and_mul) on the B200.

Numerics are checked against a plain PyTorch fp32 reference of the same op
(fp32 inputs from the same bf16 values, fp32 accumulate): the bf16 outputs
may differ from the rounded reference by one bf16 ulp where the accumulation
order moves a value across a rounding boundary.  The fused gate/up kernel is
checked bit-for-bit against mm followed by silu_and_mul.
"""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _m():
    import torch_mcpu_b200

    return torch_mcpu_b200


def rand_bf16(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).to(torch.bfloat16).to(DEV)


def check_close(out, ref32):
    ref = ref32.to(torch.bfloat16).float()
    o = out.float()
    err = (o - ref32).norm() / ref32.norm()
    assert err < 5e-3, float(err)
    tol = ref.abs() * (2.0 ** -7) + 1e-3 * ref32.abs().max()
    bad = ((o - ref).abs() > tol).sum().item()
    assert bad == 0, f"{bad} elements beyond one bf16 ulp"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (77, 296, 200), (1, 256, 64),
                                   (300, 1000, 4096), (2048, 4096, 4096), (129, 8, 72)])
def test_mm_matches_fp32_reference(M, N, K):
    a = rand_bf16(M, K, seed=1)
    b = rand_bf16(N, K, seed=2, scale=0.05)
    _m().device_error(reset=True)
    out = _m().mm_nt(a, b)
    torch.cuda.synchronize()
    assert _m().device_error() == 0
    check_close(out, a.float() @ b.float().t())


def test_addmm_matches_fp32_reference():
    M, N, K = 200, 512, 256
    a = rand_bf16(M, K, seed=3)
    b = rand_bf16(N, K, seed=4, scale=0.05)
    bias = rand_bf16(N, seed=5)
    out = _m().mm_nt(a, b, bias=bias)
    torch.cuda.synchronize()
    check_close(out, a.float() @ b.float().t() + bias.float())


def test_mm_is_deterministic_and_stream_ordered():
    a = rand_bf16(512, 1024, seed=6)
    b = rand_bf16(768, 1024, seed=7, scale=0.05)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        o1 = _m().mm_nt(a, b)
        o2 = _m().mm_nt(a, b)
    s.synchronize()
    assert torch.equal(o1, o2)


@pytest.mark.parametrize("M,I,K", [(64, 128, 64), (300, 512, 256), (2048, 1792, 4096)])
def test_gemm_swiglu_equals_mm_then_silu_and_mul(M, I, K):
    m = _m()
    x = rand_bf16(M, K, seed=8)
    wg = rand_bf16(I, K, seed=9, scale=0.05)
    wu = rand_bf16(I, K, seed=10, scale=0.05)
    w = torch.cat([wg, wu], 0)
    gu = m.mm_nt(x, w)
    ref = torch.empty(M, I, dtype=torch.bfloat16, device=DEV)
    m.silu_and_mul(ref, gu)
    fused = m.gemm_swiglu(x, m.interleave_gate_up(w))
    torch.cuda.synchronize()
    assert m.device_error() == 0
    assert torch.equal(fused, ref)
    # and the silu/mul step itself is the oracle's
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    np.testing.assert_array_equal(bits(ref), oracle.silu_and_mul_bf16(bits(gu), exp_mode=oracle.EXP_CR))


def test_mm_rejects_bad_arguments():
    m = _m()
    a = rand_bf16(16, 64)
    with pytest.raises(RuntimeError, match="must match"):
        m.mm_nt(a, rand_bf16(32, 72))
    with pytest.raises(RuntimeError, match="multiples of 8"):
        m.mm_nt(rand_bf16(16, 60), rand_bf16(32, 60))
    with pytest.raises(RuntimeError, match="bfloat16"):
        m.mm_nt(a.float(), rand_bf16(32, 64))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kernels_with_large_shared_memory_run_on_a_second_device_in_one_process():
    """The raised shared-memory limit of a kernel belongs to one device's
    context: a GEMM (over 48 KiB of shared memory), the MoE dispatch with
    1024 experts and the router, first on device 0 and then on device 1 of
    the same process, each against the same call on device 0."""
    m = _m()
    outs = []
    g = torch.Generator().manual_seed(21)
    a = (torch.randn(512, 256, generator=g)).to(torch.bfloat16)
    b = (0.05 * torch.randn(384, 256, generator=g)).to(torch.bfloat16)
    ids = torch.randint(0, 1024, (3000, 8), generator=g, dtype=torch.int32)
    logits = torch.randn(300, 256, generator=g)
    bias = 0.01 * torch.randn(256, generator=g)
    for d in (0, 1):
        dev = f"cuda:{d}"
        with torch.cuda.device(d):
            y = m.ops.mm_nt(a.to(dev), b.to(dev))
            s, e, n = m.ops.moe_align_block_size(ids.to(dev), 32, 1024)
            w, i = m.grouped_topk(logits.to(dev), logits.to(dev), 8, True, 8, 4, "sigmoid", 2.5, bias.to(dev))
            torch.cuda.synchronize(d)
            outs.append([t.cpu() for t in (y, s, e, n, w, i)])
    for x0, x1 in zip(*outs):
        assert torch.equal(x0, x1)
