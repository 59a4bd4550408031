"""The mcpu PyTorch device on B200.

    import torch_mcpu_b200.device          # once, before any mcpu tensor
    x = torch.randn(4, 8).to("mcpu")

Mirrors what `import torch_mcpu` does in the reference
(torch_mcpu/__init__.py:32-39): renames PrivateUse1 to "mcpu", registers the
device module `torch.mcpu` (torch_mcpu/openreg/__init__.py:439-479: device,
streams, memory, kernel timing, synchronize; the op-timing profiler hooks
and the host-view helpers of the simulated device are not part of it), generates the tensor methods
(`.mcpu()`, `.is_mcpu`) and registers the "mcpu" distributed backend
(torch_mcpu/distributed.py:11-20), here backed by NCCL.
"""

from __future__ import annotations

import importlib.util
import os
import types

import torch

from . import _lib, build_ext

_C = None


def _load_extension():
    global _C
    if _C is not None:
        return _C
    _lib.load()  # the C-ABI library the extension links against
    if not os.path.exists(build_ext.SO):
        build_ext.build()
    import torch.distributed  # noqa: F401  registers c10d's pybind types

    spec = importlib.util.spec_from_file_location(build_ext.NAME, build_ext.SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    _C = mod
    return mod


_C = _load_extension()


# ---------------------------------------------------------------- torch.mcpu
def is_available() -> bool:
    return _C._get_device_count() > 0


def device_count() -> int:
    return _C._get_device_count()


def current_device() -> int:
    return _C._get_device()


def set_device(device) -> None:
    idx = torch.device(device).index if not isinstance(device, int) else device
    if idx is not None:
        _C._set_device(idx)


def synchronize(device=None) -> None:
    idx = -1 if device is None else (device if isinstance(device, int) else torch.device(device).index)
    _C._synchronize(-1 if idx is None else idx)


def current_stream_handle(device=None) -> int:
    """The cudaStream_t behind the current mcpu stream (for the C-ABI)."""
    idx = current_device() if device is None else (device if isinstance(device, int) else torch.device(device).index)
    return _C._current_stream_handle(idx)


def _index(device) -> int:
    if device is None:
        return current_device()
    if isinstance(device, int):
        return device
    idx = torch.device(device).index
    return current_device() if idx is None else idx


class device:
    """Context manager that makes `device` current (torch.mcpu.device)."""

    def __init__(self, device):
        self.idx = -1 if device is None else _index(device)
        self.prev = -1

    def __enter__(self):
        self.prev = current_device()
        if self.idx >= 0 and self.idx != self.prev:
            _C._set_device(self.idx)

    def __exit__(self, *a):
        if self.idx >= 0 and self.idx != self.prev:
            _C._set_device(self.prev)
        return False


class Stream(torch.Stream):
    """An mcpu stream (a CUDA stream underneath)."""

    def __new__(cls, device=None, priority=0, **kwargs):
        if kwargs:
            return super().__new__(cls, priority=priority, **kwargs)
        return super().__new__(cls, device=torch.device("mcpu", _index(device)), priority=priority)


class StreamContext:
    """Selects a stream for the scope of a `with` block (no-op for None)."""

    def __init__(self, stream):
        self.stream = stream
        self.prev = None

    def __enter__(self):
        if self.stream is not None:
            self.prev = torch.accelerator.current_stream(self.stream.device)
            torch.accelerator.set_stream(self.stream)
        return self.stream

    def __exit__(self, *a):
        if self.stream is not None:
            torch.accelerator.set_stream(self.prev)
        return False


def stream(stream) -> StreamContext:
    return StreamContext(stream)


def current_stream(device=None) -> torch.Stream:
    return torch.accelerator.current_stream(torch.device("mcpu", _index(device)))


def default_stream(device=None) -> torch.Stream:
    sid, idx, dtype = _C._get_default_stream(_index(device))
    return torch.Stream(stream_id=sid, device_type=dtype, device_index=idx)


def set_stream(stream) -> None:
    if stream is not None:
        torch.accelerator.set_stream(stream)


def set_kernel_timing_enabled(enabled: bool) -> None:
    _C._set_kernel_timing_enabled(bool(enabled))


def reset_kernel_timing() -> None:
    _C._reset_kernel_timing()


def get_kernel_timing() -> list:
    """[{"role", "events": [{"name", "stream", "begin_time", "end_time",
    "elapsed_time"(us)}]}] for launches made through the launch API."""
    return _C._get_kernel_timing()


class Graph:
    """A CUDA graph of the work enqueued on the current mcpu stream.

        g = torch.mcpu.Graph()
        with torch.mcpu.stream(s), g.capture():   # a non-default stream
            step()                                 # no device allocation inside
        g.replay()

    Replays run on the current mcpu stream.  Work inside the capture must
    not allocate device memory (use preallocated outputs / out= ops); a graph
    holding collectives is reset before the process group is destroyed."""

    def __init__(self):
        self._exec = 0
        self._dev = current_device()

    def capture(self):
        graph = self

        class _Ctx:
            def __enter__(self):
                graph._dev = current_device()
                _C._graph_begin(graph._dev)
                return graph

            def __exit__(self, *a):
                graph._exec = _C._graph_end(graph._dev)
                return False

        return _Ctx()

    def replay(self):
        if not self._exec:
            raise RuntimeError("torch.mcpu.Graph: nothing captured")
        _C._graph_replay(self._exec, self._dev)

    def reset(self):
        if self._exec:
            _C._graph_destroy(self._exec)
            self._exec = 0

    def __del__(self):
        try:
            self.reset()
        except Exception:
            pass


def get_memory_info(device=None) -> tuple:
    """(free, total) bytes of the device."""
    return tuple(_C._mem_get_info(_index(device)))


mem_get_info = get_memory_info


def memory_stats(device=None) -> dict:
    idx = _index(device)
    st = dict(_C._memory_stats(idx))
    cur, peak = _C._mem_pool_reserved(idx)
    st["reserved_bytes.all.current"] = cur
    st["reserved_bytes.all.peak"] = peak
    return st


def memory_reserved(device=None) -> int:
    return memory_stats(device)["reserved_bytes.all.current"]


def max_memory_reserved(device=None) -> int:
    return memory_stats(device)["reserved_bytes.all.peak"]


def memory_allocated(device=None) -> int:
    return memory_stats(device)["allocated_bytes.all.current"]


def max_memory_allocated(device=None) -> int:
    return memory_stats(device)["allocated_bytes.all.peak"]


def reset_peak_memory_stats(device=None) -> None:
    _C._reset_peak_memory_stats(current_device() if device is None else int(device))


def empty_cache() -> None:
    _C._empty_cache()


def is_initialized() -> bool:
    return True


def init() -> None:
    pass


def manual_seed(seed: int) -> None:
    # mcpu tensors are drawn by the host generator, then copied; torch.manual_seed
    # itself calls manual_seed_all of this module, so seed the generator directly
    torch.default_generator.manual_seed(int(seed))


def manual_seed_all(seed: int) -> None:
    torch.default_generator.manual_seed(int(seed))


def _is_in_bad_fork() -> bool:
    return False


def get_rng_state(device=None):
    return torch.get_rng_state()


def set_rng_state(state, device=None):
    torch.set_rng_state(state)


_module = types.ModuleType("torch.mcpu")
for _n in ["is_available", "device_count", "current_device", "set_device", "synchronize",
           "current_stream_handle", "memory_stats", "memory_allocated", "max_memory_allocated",
           "memory_reserved", "max_memory_reserved", "get_memory_info", "mem_get_info",
           "reset_peak_memory_stats", "empty_cache", "is_initialized", "init", "manual_seed",
           "manual_seed_all", "_is_in_bad_fork", "get_rng_state", "set_rng_state", "device",
           "Stream", "StreamContext", "stream", "current_stream", "default_stream", "set_stream",
           "set_kernel_timing_enabled", "reset_kernel_timing", "get_kernel_timing", "Graph"]:
    setattr(_module, _n, globals()[_n])


def _setup():
    if torch._C._get_privateuse1_backend_name() != "mcpu":
        torch.utils.rename_privateuse1_backend("mcpu")
    if not hasattr(torch, "mcpu"):
        torch._register_device_module("mcpu", _module)
        torch.utils.generate_methods_for_privateuse1_backend(for_storage=True)
    import torch.distributed as dist

    if dist.is_available() and not dist.is_backend_available("mcpu"):
        dist.Backend.register_backend("mcpu", _C.create_process_group_mcpu, devices=["mcpu"])


_setup()
