"""Host side of mcpu_grouped_topk_moe_align, without a device: the workspace
size, and the argument errors it returns before anything is enqueued (the
reference-style message in mcpuGetLastErrorString)."""

import ctypes

import pytest


def _lib():
    from torch_mcpu_b200 import _lib

    return _lib.load()


def _ws_bytes(lib, T, E, K):
    n = ctypes.c_uint64()
    rc = lib.mcpu_grouped_topk_moe_align_workspace_bytes(T, E, K, ctypes.byref(n))
    return rc, n.value


def test_workspace_covers_the_two_launch_path_and_grows_with_the_batch():
    lib = _lib()
    rc, fused = _ws_bytes(lib, 65536, 256, 8)
    assert rc == 0
    moe = ctypes.c_uint64()
    assert lib.mcpu_moe_align_workspace_bytes(65536 * 8, 256, ctypes.byref(moe)) == 0
    # header (generation, arrival counts, group sums) + the larger of the rows
    # and the two-launch path's count matrix
    assert fused >= 128 + moe.value
    rc, big = _ws_bytes(lib, 1 << 20, 256, 8)
    assert rc == 0 and big >= fused
    rc, empty = _ws_bytes(lib, 0, 256, 8)
    assert rc == 0 and empty > 0


@pytest.mark.parametrize("T,E,K", [(-1, 256, 8), (1 << 28, 256, 8), (16, 256, 0), (16, 256, 17)])
def test_workspace_size_rejects_out_of_range_shapes(T, E, K):
    rc, _ = _ws_bytes(_lib(), T, E, K)
    assert rc != 0


def _call(lib, **kw):
    a = dict(gating=1 << 20, dtype=0, T=64, E=256, G=8, TG=4, K=8, renorm=1, scale=2.5, bias=1 << 21,
             scoring=1, w=1 << 22, ids=1 << 23, bs=64, sorted=1 << 24, cap=64 * 8 + 256 * 63,
             eids=1 << 25, ecap=(64 * 8 + 256 * 63 + 63) // 64, npad=1 << 26, ws=1 << 27, wsb=1 << 30,
             stream=None)
    a.update(kw)
    return lib.mcpu_grouped_topk_moe_align(a["gating"], a["dtype"], a["T"], a["E"], a["G"], a["TG"], a["K"],
                                           a["renorm"], a["scale"], a["bias"], a["scoring"], a["w"], a["ids"],
                                           a["bs"], a["sorted"], a["cap"], a["eids"], a["ecap"], a["npad"],
                                           a["ws"], a["wsb"], a["stream"])


@pytest.mark.parametrize("kw,msg", [
    ({"E": 250}, b"divisible"),
    ({"K": 0}, b"topk"),
    ({"dtype": 7}, b"float32 or bfloat16"),
    ({"cap": 16}, b"sorted_token_ids holds"),
    ({"ecap": 1}, b"expert_ids holds"),
    ({"bs": 0}, b"block_size"),
    ({"npad": None}, b"NULL"),
    ({"wsb": 8}, b"workspace of"),
    ({"ws": (1 << 27) + 4}, b"workspace of"),
])
def test_argument_errors_before_any_launch(kw, msg):
    lib = _lib()
    assert _call(lib, **kw) != 0
    assert msg in lib.mcpuGetLastErrorString()
