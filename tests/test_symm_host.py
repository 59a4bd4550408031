"""Host logic of the symmetric windows behind mcpu_mm_allreduce, without a GPU:
the window sizing of the C-ABI (pure host functions of the device library),
and the IPC-handle exchange through the process group's store between two
gloo ranks, with the device calls replaced by a fake that hands out
recognisable pointers."""

import ctypes
import os
import tempfile

import pytest
import torch


def _lib():
    from torch_mcpu_b200 import _lib as L

    return L, L.load()


def _window_bytes(lib, M, N, world):
    v = ctypes.c_uint64()
    assert lib.mcpu_mm_allreduce_window_bytes(M, N, world, ctypes.byref(v)) == 0
    return v.value


def _control_bytes(lib, nbytes, world):
    v = ctypes.c_uint64()
    assert lib.mcpu_mm_allreduce_control_bytes(nbytes, world, ctypes.byref(v)) == 0
    return v.value


@pytest.mark.parametrize("M,N,world", [(1, 256, 1), (2048, 4096, 8), (1000, 4096, 2), (8192, 7168, 4),
                                       (256, 7168, 8), (4097, 512, 3)])
def test_window_holds_control_slots_and_output(M, N, world):
    L, lib = _lib()
    nbytes = _window_bytes(lib, M, N, world)
    ctrl = _control_bytes(lib, nbytes, world)
    tiles = -(-M // 128) * (N // 256)
    slices = tiles * 4
    slots = -(-slices // world)
    assert ctrl % 4096 == 0 and ctrl >= 256 + 4 * 4 * slots  # done word, then one counter per unit
    recv = world * slots * 32 * 256 * 2
    assert nbytes >= ctrl + recv + M * N * 2
    assert nbytes % 4096 == 0
    # a window sized for this problem also holds every smaller M
    assert _window_bytes(lib, max(1, M // 2), N, world) <= nbytes


def test_window_sizing_rejects_bad_arguments():
    L, lib = _lib()
    v = ctypes.c_uint64()
    assert lib.mcpu_mm_allreduce_window_bytes(128, 300, 2, ctypes.byref(v)) != 0
    assert lib.mcpu_mm_allreduce_window_bytes(128, 256, 9, ctypes.byref(v)) != 0
    assert lib.mcpu_mm_allreduce_control_bytes(1 << 20, 0, ctypes.byref(v)) != 0


class _FakeLib:
    """Device calls of SymmetricWindow: rank r's window is 0x10000000*(r+1);
    opening rank q's handle maps it at 0x7000000000 + 0x100000*q."""

    def __init__(self, rank):
        self.rank, self.closed, self.freed = rank, [], []

    def mcpu_symm_alloc(self, nbytes, pptr, handle):
        pptr._obj.value = 0x10000000 * (self.rank + 1)
        for i in range(len(handle)):
            handle[i] = (self.rank * 31 + i) & 0xFF
        return 0

    def mcpu_symm_open(self, handle, pptr):
        q = handle[0] // 31
        assert all(handle[i] == (q * 31 + i) & 0xFF for i in range(len(handle)))
        pptr._obj.value = 0x7000000000 + 0x100000 * q
        return 0

    def mcpu_symm_close(self, p):
        self.closed.append(p)
        return 0

    def mcpu_symm_free(self, p):
        self.freed.append(p)
        return 0


def _exchange_worker(rank, world, path, q):
    try:
        import types

        import torch.distributed as dist

        from torch_mcpu_b200 import _lib as L
        from torch_mcpu_b200 import symm

        fake = _FakeLib(rank)
        L.load = lambda *a, **k: fake
        torch.mcpu = types.SimpleNamespace(current_device=lambda: 0, synchronize=lambda *a: None)
        store = dist.FileStore(path, world)
        w1 = symm.SymmetricWindow(1 << 20, rank=rank, world=world, store=store)
        w2 = symm.SymmetricWindow(1 << 21, rank=rank, world=world, store=store)
        b1, b2 = w1.bases(), w2.bases()
        h = w1.handle
        w1.close()
        w2.close()
        q.put((rank, b1, b2, h != 0, fake.closed, fake.freed))
    except Exception:  # pragma: no cover - reported to the parent
        import traceback

        q.put((rank, traceback.format_exc()))


def test_handle_exchange_through_the_store_two_ranks():
    import torch.multiprocessing as mp

    world = 2
    fd, path = tempfile.mkstemp(prefix="mcpu_symm_")
    os.close(fd)
    os.unlink(path)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, path, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        item = q.get(timeout=120)
        res[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert len(res[r]) == 5, res[r][0]
        b1, b2, has_handle, closed, freed = res[r]
        want = [0x10000000 * (r + 1) if q == r else 0x7000000000 + 0x100000 * q for q in range(world)]
        assert b1 == want and b2 == want
        assert has_handle
        peers = [0x7000000000 + 0x100000 * q for q in range(world) if q != r]
        assert closed == peers * 2  # every mapped peer window unmapped, per window
        assert freed == [0x10000000 * (r + 1)] * 2
