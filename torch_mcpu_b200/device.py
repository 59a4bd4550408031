"""The mcpu PyTorch device on B200.

    import torch_mcpu_b200.device          # once, before any mcpu tensor
    x = torch.randn(4, 8).to("mcpu")

Mirrors what `import torch_mcpu` does in the reference
(torch_mcpu/__init__.py:32-39): renames PrivateUse1 to "mcpu", registers the
device module `torch.mcpu` (torch_mcpu/openreg/__init__.py:439-479 subset:
device/stream/memory/synchronize), generates the tensor methods
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


def memory_stats(device=None) -> dict:
    return dict(_C._memory_stats(current_device() if device is None else int(device)))


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
    torch.manual_seed(seed)  # mcpu tensors are drawn on the host, then copied


def manual_seed_all(seed: int) -> None:
    torch.manual_seed(seed)


def _is_in_bad_fork() -> bool:
    return False


def get_rng_state(device=None):
    return torch.get_rng_state()


def set_rng_state(state, device=None):
    torch.set_rng_state(state)


_module = types.ModuleType("torch.mcpu")
for _n in ["is_available", "device_count", "current_device", "set_device", "synchronize",
           "current_stream_handle", "memory_stats", "memory_allocated", "max_memory_allocated",
           "reset_peak_memory_stats", "empty_cache", "is_initialized", "init", "manual_seed",
           "manual_seed_all", "_is_in_bad_fork", "get_rng_state", "set_rng_state"]:
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
