"""Symmetric windows over CUDA IPC, and the fused down projection +
all-reduce that runs in them.

A SymmetricWindow is one device buffer of the same size on every rank of a
tensor-parallel group (one process per GPU of one box).  Each rank allocates
its own (mcpu_symm_alloc), publishes the IPC handle in the process group's
store and maps every other rank's buffer (mcpu_symm_open), so a kernel can
store into and load from the peers' windows over NVLink.  The reference has
no counterpart: its ProcessGroup copies tensors through host memory
(torch_mcpu/csrc/Distributed.cpp:281-354).

mm_allreduce(a, b, window) is mm(a, b.t()) followed by a SUM all-reduce
over the group, as the reference's TP MLP step runs them
(example/01_mlp_tp4/run.py:106-113), in one kernel.
"""

from __future__ import annotations

import ctypes
import itertools
import time

import torch

from . import _lib

_SEQ = itertools.count()


def _store_barrier(store, key: str, world: int, timeout_s: float) -> None:
    store.add(key, 1)
    deadline = time.monotonic() + timeout_s
    while int(store.add(key, 0)) < world:
        if time.monotonic() > deadline:
            raise RuntimeError(f"symmetric window: ranks did not reach {key} within {timeout_s} s")
        time.sleep(0.001)


class SymmetricWindow:
    """`nbytes` of device memory on every rank, mapped by all ranks.

    With torch.distributed initialised, rank and world come from the default
    group and the IPC handles travel through its store; every rank must
    create its windows in the same order.  Without it (or with world=1) the
    window is local to this process.  Windows are created on the current
    mcpu device."""

    def __init__(self, nbytes: int, *, rank: int | None = None, world: int | None = None, store=None,
                 timeout_s: float = 120.0):
        import torch.distributed as dist

        if world is None:
            if dist.is_available() and dist.is_initialized():
                rank, world = dist.get_rank(), dist.get_world_size()
            else:
                rank, world = 0, 1
        if rank is None:
            raise RuntimeError("SymmetricWindow: rank is required with world")
        if not 1 <= world <= _lib.SYMM_MAX_RANKS:
            raise RuntimeError(f"SymmetricWindow: world {world} outside 1..{_lib.SYMM_MAX_RANKS}")
        if world > 1 and store is None:
            store = dist.distributed_c10d._get_default_store()
        self.rank, self.world, self.nbytes = rank, world, int(nbytes)
        self.device = torch.mcpu.current_device()
        self._store, self._timeout = store, timeout_s
        self._key = f"mcpu_symm/{next(_SEQ)}"
        lib = _lib.load()
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.SYMM_HANDLE_BYTES)()
        _lib.check(lib.mcpu_symm_alloc(self.nbytes, ctypes.byref(ptr), handle), "symm_alloc")
        bases = [0] * world
        bases[rank] = ptr.value
        self._opened: list[int] = []
        try:
            if world > 1:
                store.set(f"{self._key}/{rank}", bytes(handle))
                for r in range(world):
                    if r == rank:
                        continue
                    h = store.get(f"{self._key}/{r}")
                    if len(h) != _lib.SYMM_HANDLE_BYTES:
                        raise RuntimeError(f"SymmetricWindow: bad handle from rank {r}")
                    hb = (ctypes.c_uint8 * _lib.SYMM_HANDLE_BYTES).from_buffer_copy(h)
                    p = ctypes.c_void_p()
                    _lib.check(lib.mcpu_symm_open(hb, ctypes.byref(p)), f"symm_open (rank {r})")
                    bases[r] = p.value
                    self._opened.append(p.value)
        except Exception:
            for p in self._opened:
                lib.mcpu_symm_close(p)
            lib.mcpu_symm_free(ptr.value)
            raise
        arr = (ctypes.c_void_p * _lib.SYMM_MAX_RANKS)(*(bases + [None] * (_lib.SYMM_MAX_RANKS - world)))
        self._win = _lib.SymmWindow(rank, world, self.nbytes, arr)
        self._local = ptr.value

    @property
    def handle(self) -> int:
        """Address of the mcpuSymmWindow (the `window` argument of the ops)."""
        if self._win is None:
            raise RuntimeError("SymmetricWindow is closed")
        return ctypes.addressof(self._win)

    def bases(self) -> list[int]:
        return [int(self._win.base[r] or 0) for r in range(self.world)]

    def control_bytes(self) -> int:
        v = ctypes.c_uint64()
        _lib.check(_lib.load().mcpu_mm_allreduce_control_bytes(self.nbytes, self.world, ctypes.byref(v)),
                   "mm_allreduce_control_bytes")
        return int(v.value)

    def clear_counters(self) -> None:
        """Zero this rank's counters (after a call that failed on any rank;
        every rank clears its own, then the group synchronises)."""
        torch.mcpu.synchronize()
        _lib.check(_lib.load().mcpu_symm_clear(self._local, self.control_bytes(), None), "symm_clear")
        torch.mcpu.synchronize()
        if self.world > 1:
            _store_barrier(self._store, f"{self._key}/clear/{next(_SEQ)}", self.world, self._timeout)

    def close(self) -> None:
        """Collective: unmaps the peers' windows and frees this one once no
        rank can still write to it."""
        if self._win is None:
            return
        lib = _lib.load()
        torch.mcpu.synchronize()
        if self.world > 1:
            _store_barrier(self._store, f"{self._key}/close", self.world, self._timeout)
        for p in self._opened:
            lib.mcpu_symm_close(p)
        if self.world > 1:
            _store_barrier(self._store, f"{self._key}/closed", self.world, self._timeout)
        lib.mcpu_symm_free(self._local)
        self._win = None


def window_bytes(M: int, N: int, world: int) -> int:
    """Window size mm_allreduce needs for an [M, N] output over `world` ranks."""
    v = ctypes.c_uint64()
    _lib.check(_lib.load().mcpu_mm_allreduce_window_bytes(M, N, world, ctypes.byref(v)),
               "mm_allreduce_window_bytes")
    return int(v.value)


def mm_allreduce(a: torch.Tensor, b: torch.Tensor, window: SymmetricWindow) -> torch.Tensor:
    """sum over ranks of a_r @ b_r.T (bf16, [M, N]) on every rank, in one
    kernel: the tensor-core epilogue sends each slice of the partial to its
    owner rank, which sums the partials in fp32 in rank order and writes the
    bf16 result to every rank.  Returns a view of this rank's window, valid
    until the next mm_allreduce on `window`."""
    return torch.ops.mcpu.mm_allreduce(a, b, window.handle)
