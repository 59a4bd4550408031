"""mcpu_moe_align_block_size_static: MoE dispatch for callers that cannot
allocate device memory when they dispatch experts (an engine whose memory
pool already holds all free device memory, serving code that must not stall
on cudaMalloc, C callers with no device allocator).  It keeps its counters
in a fixed array of the library's device memory instead of a workspace.

Called through the C-ABI, twice in a row with different inputs (the second
call finds the first call's counters in the shared array), and checked
against the workspace entry point, mcpu_moe_align_block_size: integer
outputs, so they must be identical.  Also: a problem beyond the array's
limit is refused with a message naming it.  This file is collected last so
that a run stopping at its first failure has run every other test before."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _outputs(numel, E, bs):
    cap = min(numel + E * (bs - 1), numel * bs)
    nblk = -(-cap // bs)
    return (torch.empty(cap, dtype=torch.int32, device="cuda"), torch.empty(nblk, dtype=torch.int32, device="cuda"),
            torch.empty(1, dtype=torch.int32, device="cuda"))


def _with_workspace(lib, ids, E, bs, stream):
    from torch_mcpu_b200 import _lib

    s, e, n = _outputs(ids.numel(), E, bs)
    ws = ctypes.c_uint64()
    _lib.check(lib.mcpu_moe_align_workspace_bytes(ids.numel(), E, ctypes.byref(ws)), "workspace bytes")
    work = torch.empty(ws.value, dtype=torch.uint8, device="cuda")
    _lib.check(lib.mcpu_moe_align_block_size(ids.data_ptr(), ids.numel(), E, bs, s.data_ptr(), s.numel(),
                                             e.data_ptr(), e.numel(), n.data_ptr(), work.data_ptr(), ws.value,
                                             stream), "moe_align_block_size")
    torch.cuda.synchronize()
    return s.cpu(), e.cpu(), n.cpu()


def _static(lib, ids, E, bs, stream):
    from torch_mcpu_b200 import _lib

    s, e, n = _outputs(ids.numel(), E, bs)
    _lib.check(lib.mcpu_moe_align_block_size_static(ids.data_ptr(), ids.numel(), E, bs, s.data_ptr(), s.numel(),
                                                    e.data_ptr(), e.numel(), n.data_ptr(), stream),
               "moe_align_block_size_static")
    torch.cuda.synchronize()
    return s.cpu(), e.cpu(), n.cpu()


def test_static_scratch_entry_point_matches_the_workspace_one_on_two_calls():
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    g = np.random.default_rng(11)
    # router-sized call (65536 tokens, top-8 of 256 experts, block 64), then a
    # smaller one with another expert count: the second call reuses the array
    cases = [(g.integers(0, 256, (65536, 8)), 256, 64), (g.integers(0, 160, (1000, 6)), 160, 16)]
    _check_cases(lib, stream, cases)


def _check_cases(lib, stream, cases):
    for ids_np, E, bs in cases:
        ids = torch.from_numpy(ids_np.astype(np.int32)).cuda()
        want = _with_workspace(lib, ids, E, bs, stream)
        got = _static(lib, ids, E, bs, stream)
        for a, b in zip(got, want):
            assert torch.equal(a, b)


def test_static_scratch_entry_point_at_its_limit_and_after_a_larger_matrix():
    """Exactly at the limit (256 chunks x 256 experts = 65536 counters), then
    a small call with 1024 experts whose count matrix is a different shape
    than the counters the previous call left in the array."""
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    g = np.random.default_rng(12)
    cases = [(g.integers(0, 256, (4096 * 256,)), 256, 64), (g.integers(0, 1024, (3000, 8)), 1024, 32)]
    _check_cases(lib, stream, cases)


def test_static_scratch_entry_point_refuses_problems_beyond_its_limit():
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    ids = torch.zeros(8, dtype=torch.int32, device="cuda")
    out = torch.zeros(8, dtype=torch.int32, device="cuda")
    numel = 4096 * 257  # 257 chunks x 256 experts > 65536 counters; refused before any launch
    rc = lib.mcpu_moe_align_block_size_static(ids.data_ptr(), numel, 256, 64, out.data_ptr(), out.numel(),
                                              out.data_ptr(), out.numel(), out.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc != 0
    assert b"fixed scratch holds 65536" in lib.mcpuGetLastErrorString()
