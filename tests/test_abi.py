"""The C-ABI library loads and exports every entry point include/*.h declares.

CPU only: nothing here launches device work.
"""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = "\n".join(line for line in src.splitlines() if not line.lstrip().startswith("#"))
        for m in re.finditer(r"OPENREG_EXPORT\s+[^;(]*?\b(\w+)\s*\(", src):
            names.append(m.group(1))
    return names


def test_headers_declare_entry_points():
    names = declared_symbols()
    assert "orMalloc" in names and "mcpu_grouped_topk" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_every_declared_symbol():
    from torch_mcpu_b200 import _lib

    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_error_string_and_argument_validation_without_device():
    """Argument checks run on the host before any device call."""
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    rc = lib.mcpu_grouped_topk(None, 0, 4, 12, 8, 1, 2, 1, 1.0, None, 0, None, None, None)
    assert rc == 4  # orErrorInvalidValue
    assert b"divisible" in lib.mcpuGetLastErrorString()
    rc = lib.mcpu_grouped_topk(None, 0, 0, 256, 8, 4, 8, 1, 1.0, None, 1, None, None, None)
    assert rc == 0  # zero tokens: nothing to do


def test_priority_range_matches_reference_convention():
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    lo, hi = ctypes.c_int(-9), ctypes.c_int(-9)
    assert lib.orDeviceGetStreamPriorityRange(ctypes.byref(lo), ctypes.byref(hi)) == 0
    assert (lo.value, hi.value) == (1, 0)


def test_memory_protection_calls_are_accepted():
    from torch_mcpu_b200 import _lib

    lib = _lib.load()
    assert lib.orMemoryProtect(None) == 0 and lib.orMemoryUnprotect(None) == 0


def test_extension_exports_the_launch_api():
    """include/mcpu_launch.h's exported functions (kernel timing, guards,
    stream lookups) are defined by the PyTorch-facing extension."""
    import subprocess

    from torch_mcpu_b200 import build_ext

    if not os.path.exists(build_ext.SO):
        pytest.skip("extension not built")
    src = open(os.path.join(ROOT, "include", "mcpu_launch.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = "\n".join(line for line in src.splitlines() if not line.lstrip().startswith("#"))
    wanted = set(re.findall(r"MCPU_LAUNCH_EXPORT\s+(?:extern\s+)?[\w:<>\s\*&]*?\b(\w+)\s*[\(;]", src))
    assert {"getCurrentMcpuStream", "reserve_event_slot", "get_kernel_launch_stream", "g_enabled"} <= wanted
    out = subprocess.run(["nm", "-DC", "--defined-only", build_ext.SO], capture_output=True, text=True).stdout
    missing = [w for w in wanted if not re.search(r"\b" + w + r"\b", out)]
    assert not missing, missing


def test_extension_shares_libstdcxx_with_torch():
    """The torch extension must use the process's libstdc++ (dynamically),
    not a private static copy: torch formats its error messages with its own
    streams, and a second copy of the stream code crashes on them."""
    import shutil
    import subprocess

    from torch_mcpu_b200 import build_ext

    if shutil.which("readelf") is None:
        pytest.skip("readelf not available")
    so = build_ext.build()
    dyn = subprocess.run(["readelf", "-d", so], capture_output=True, text=True).stdout
    assert "libstdc++.so" in dyn
    syms = subprocess.run(["readelf", "--dyn-syms", "-W", so], capture_output=True, text=True).stdout
    assert "_ZNKSt19__codecvt_utf8_baseIwE10do_unshift" not in syms  # libstdc++ internals not linked in
