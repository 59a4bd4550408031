"""The fused row-parallel down projection + SUM all-reduce (mcpu_mm_allreduce)
on one GPU, as a group of one rank.  The kernel runs its whole protocol
there — each slice of the partial sent to its owner's slot, the unit
counters, the owner's reduction, the done counter — through local memory,
so the result must carry the plain GEMM's bits.  Calls in a row (the
counters are reset by the kernel itself), a smaller ragged M in the same
window, the TP MLP step against the oracle, and argument errors.  The
multi-rank form is covered by tests/test_distributed_gpu.py."""

import numpy as np
import pytest
import torch

import configs as C
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def symm():
    import torch_mcpu_b200.device  # noqa: F401
    from torch_mcpu_b200 import symm as s

    assert torch.mcpu.is_available()
    return s


def _inputs(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (0.02 * torch.randn(N, K, generator=g)).to(torch.bfloat16)
    return a.to("mcpu"), b.to("mcpu")


def test_single_rank_result_is_the_gemm(symm):
    from torch_mcpu_b200 import ops

    M, N, K = 2048, 4096, 1792  # the down projection of one rank at TP=8
    win = symm.SymmetricWindow(symm.window_bytes(M, N, 1))
    try:
        for seed in (1, 2):
            a, b = _inputs(M, N, K, seed)
            y = symm.mm_allreduce(a, b, win)
            assert y.device.type == "mcpu" and tuple(y.shape) == (M, N)
            got = y.cpu()  # copied before the next call reuses the window
            ref = torch.mm(a, b.t()).cpu()
            assert torch.equal(got, ref), f"seed {seed}"
        a, b = _inputs(1000, N, 520, 3)  # ragged M and K in the same window
        got = symm.mm_allreduce(a, b, win).cpu()
        assert torch.equal(got, torch.mm(a, b.t()).cpu())
        torch.mcpu.synchronize()
        assert ops.device_error() == 0
    finally:
        win.close()


def test_single_rank_tp_step_against_oracle(symm):
    from torch_mcpu_b200 import ops
    from torch_mcpu_b200.mlp import mcpu_tp_step

    cfg = C.MLP_TINY
    x, _, wgu, wd = C.mlp_weights(cfg, 1, 0)
    xm, wgum, wdm = x.to("mcpu"), ops.interleave_gate_up(wgu).to("mcpu"), wd.to("mcpu")
    act = torch.empty(cfg.T, cfg.I, dtype=torch.bfloat16, device="mcpu")
    win = symm.SymmetricWindow(symm.window_bytes(cfg.T, cfg.H, 1))
    try:
        fused = mcpu_tp_step(xm, wgum, wdm, act, window=win).cpu()
        plain = mcpu_tp_step(xm, wgum, wdm, act).cpu()
    finally:
        win.close()
    assert torch.equal(fused, plain)
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    ref = oracle.bf16_bits_to_f32(oracle.tp_mlp_bf16(bits(x), [bits(wgu)], [bits(wd)], None,
                                                     exp_mode=oracle.EXP_CR))
    got = fused.float().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) < 2e-2


def test_argument_errors(symm):
    win = symm.SymmetricWindow(symm.window_bytes(256, 512, 1))
    try:
        a = torch.zeros(256, 64, dtype=torch.bfloat16, device="mcpu")
        with pytest.raises(RuntimeError, match="multiple of 256"):
            symm.mm_allreduce(a, torch.zeros(300, 64, dtype=torch.bfloat16, device="mcpu"), win)
        with pytest.raises(RuntimeError, match="window holds"):
            symm.mm_allreduce(torch.zeros(4096, 64, dtype=torch.bfloat16, device="mcpu"),
                              torch.zeros(512, 64, dtype=torch.bfloat16, device="mcpu"), win)
        with pytest.raises(RuntimeError, match="bfloat16"):
            symm.mm_allreduce(a.float(), torch.zeros(512, 64, device="mcpu"), win)
    finally:
        win.close()
