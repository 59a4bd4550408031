"""The reference's vLLM sampler ops (mcpu::vllm_min_p_kernel,
vllm_topk_log_softmax_kernel, vllm_ranks_kernel; csrc/aten/vllm_kernels/
min_p.cpp, logprob.cpp) on the B200 against the oracle, called as the
reference's users call them (torch.ops.mcpu on mcpu tensors): fp32, fp16
and bf16 logits, vocabularies with 16-byte-aligned and unaligned rows, a
row stride wider than the vocabulary, -inf and NaN entries, p = 0 rows and
out-of-range ids.  ranks are exact; log-probabilities within 2e-6; min_p
results identical except where an entry lies within one fp32 ulp of the
threshold (the threshold's logarithm is rounded once from fp64)."""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@pytest.fixture(scope="module")
def mcpu():
    import torch_mcpu_b200.device  # noqa: F401

    assert torch.mcpu.is_available()


def _logits(rows, width, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = (3.0 * torch.randn(rows, width, generator=g)).to(dtype)
    x[0, 5] = float("-inf")
    if rows > 1:
        x[1, 7] = float("nan")
    return x


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,width,vocab", [(7, 32000, 32000), (5, 151937, 151937), (4, 50016, 50000)])
def test_min_p(mcpu, dtype, rows, width, vocab):
    x = _logits(rows, width, dtype, 1)
    idx = torch.tensor([(3 * t) % 4 for t in range(rows)], dtype=torch.int32)
    mp = torch.tensor([0.0, 0.05, 0.3, 1e-4], dtype=torch.float32)
    xm = x.to("mcpu")
    torch.ops.mcpu.vllm_min_p_kernel(xm, idx.to("mcpu"), mp.to("mcpu"), vocab)
    got = xm.cpu().float().numpy()
    want = oracle.vllm_min_p(x.float().numpy(), idx.numpy(), mp.numpy(), vocab)
    diff = ~((got == want) | (np.isnan(got) & np.isnan(want)))
    if diff.any():
        # only entries within one fp32 ulp of their row's threshold may differ
        xf = x.float().numpy()
        for r, c in zip(*np.nonzero(diff)):
            p = mp[idx[r]].item()
            thr = np.float32(np.nanmax(xf[r, :vocab]) + np.float32(np.log(np.float64(p))))
            assert abs(xf[r, c] - thr) <= np.spacing(np.float32(thr)), (r, c)
    assert diff.sum() <= 2


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,width,vocab", [(6, 32000, 32000), (3, 151937, 151937), (4, 50016, 50000)])
def test_topk_log_softmax_and_ranks(mcpu, dtype, rows, width, vocab):
    x = _logits(rows, width, dtype, 2)
    x[1, 7] = 0.0  # a row with NaN has a NaN log-sum-exp on both sides; keep rows finite here
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, vocab, (rows, 5), generator=g)
    ids[0, 0], ids[0, 1] = -3, vocab + 10  # clamped by the op
    out = torch.empty(rows, 5, dtype=torch.float32, device="mcpu")
    torch.ops.mcpu.vllm_topk_log_softmax_kernel(out, x.to("mcpu"), ids.to("mcpu"), 5, vocab)
    want = oracle.vllm_topk_log_softmax(x.float().numpy(), ids.numpy(), vocab)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=2e-6, atol=2e-6)

    tok = ids[:, 2].clone()
    rk = torch.empty(rows, dtype=torch.int64, device="mcpu")
    torch.ops.mcpu.vllm_ranks_kernel(rk, x.to("mcpu"), tok.to("mcpu"), vocab)
    np.testing.assert_array_equal(rk.cpu().numpy(), oracle.vllm_ranks(x.float().numpy(), tok.numpy(), vocab))


def test_argument_errors(mcpu):
    x = torch.zeros(2, 8, device="mcpu")
    with pytest.raises(RuntimeError, match="vocab_size"):
        torch.ops.mcpu.vllm_min_p_kernel(x, torch.zeros(2, dtype=torch.int32, device="mcpu"),
                                         torch.zeros(1, device="mcpu"), 9)
    with pytest.raises(RuntimeError, match="float32, float16, or bfloat16"):
        torch.ops.mcpu.vllm_ranks_kernel(torch.zeros(2, dtype=torch.int64, device="mcpu"),
                                         torch.zeros(2, 8, dtype=torch.int32, device="mcpu"),
                                         torch.zeros(2, dtype=torch.int64, device="mcpu"), 8)
