"""Build and load the sm_100a native library ``koochak_b200_C``.

The library is compiled in-tree (``koochak_b200/csrc/_build/``) so that the
shared object travels with the source tree to a GPU host; nothing is written
to a user cache. ``build()`` compiles (ninja, incremental); ``load()`` imports
the already-built shared object without ever invoking the compiler, so a GPU
process never pays for, or races on, a rebuild.

``build(debug_bounds=True)`` compiles the same sources with
``-DKB_DEBUG_BOUNDS`` into ``csrc/_build_debug/koochak_b200_C_debug``: every
GEMM epilogue tile, gradient-sync chunk and sharded-Adam work item is checked
against the extent the host declared for its buffer, and a failure skips the
access and records a status code with the site and index instead of
trapping. A process loads that variant instead of the normal one when
``KOOCHAK_DEBUG_BOUNDS=1`` is set in its environment.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from types import ModuleType
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
CSRC_DIR = os.path.join(_HERE, "csrc")
BUILD_DIR = os.path.join(CSRC_DIR, "_build")
MODULE_NAME = "koochak_b200_C"
SO_PATH = os.path.join(BUILD_DIR, MODULE_NAME + ".so")
DEBUG_BUILD_DIR = os.path.join(CSRC_DIR, "_build_debug")
DEBUG_MODULE_NAME = "koochak_b200_C_debug"
DEBUG_SO_PATH = os.path.join(DEBUG_BUILD_DIR, DEBUG_MODULE_NAME + ".so")


def debug_bounds_requested() -> bool:
    return os.environ.get("KOOCHAK_DEBUG_BOUNDS", "0") not in ("", "0")

CUDA_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
    "-DNDEBUG",
]

_module: Optional[ModuleType] = None


def sources() -> list[str]:
    names = sorted(n for n in os.listdir(CSRC_DIR) if n.endswith((".cu", ".cpp")))
    return [os.path.join(CSRC_DIR, n) for n in names]


def build(verbose: bool = False, debug_bounds: bool = False) -> ModuleType:
    """Compile every CUDA source for sm_100a into ``csrc/_build`` (or the debug-bounds variant) and import it."""

    global _module
    build_dir = DEBUG_BUILD_DIR if debug_bounds else BUILD_DIR
    os.makedirs(build_dir, exist_ok=True)
    from torch.utils.cpp_extension import load

    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    defines = ["-DKB_DEBUG_BOUNDS"] if debug_bounds else []
    mod = load(
        name=DEBUG_MODULE_NAME if debug_bounds else MODULE_NAME,
        sources=sources(),
        build_directory=build_dir,
        extra_cflags=["-O3", "-std=c++17"] + defines,
        extra_cuda_cflags=list(CUDA_FLAGS) + defines,
        extra_include_paths=[CSRC_DIR],
        extra_ldflags=[],
        verbose=verbose,
    )
    if debug_bounds == debug_bounds_requested():
        _module = mod
    return mod


def load() -> ModuleType:
    """Import the prebuilt library; raise ImportError if it has not been built."""

    global _module
    if _module is not None:
        return _module
    name, path = (DEBUG_MODULE_NAME, DEBUG_SO_PATH) if debug_bounds_requested() else (MODULE_NAME, SO_PATH)
    if name in sys.modules:
        _module = sys.modules[name]
        return _module
    if not os.path.exists(path):
        raise ImportError(
            f"koochak_b200 native library not built ({path} missing); "
            "run `python -c 'import __graft_entry__ as g; g.build()'` or koochak_b200._native_build.build()"
        )
    import torch  # noqa: F401  (the extension links against torch's libraries)

    spec = importlib.util.spec_from_file_location(name, path)
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[name] = mod
    _module = mod
    return mod


if __name__ == "__main__":
    dbg = "--debug-bounds" in sys.argv
    build(verbose="-v" in sys.argv, debug_bounds=dbg)
    print(DEBUG_SO_PATH if dbg else SO_PATH)
