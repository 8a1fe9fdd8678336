"""Build and load the sm_100a native library ``koochak_b200_C``.

The library is compiled in-tree (``koochak_b200/csrc/_build/``) so that the
shared object travels with the source tree to a GPU host; nothing is written
to a user cache. ``build()`` compiles (ninja, incremental); ``load()`` imports
the already-built shared object without ever invoking the compiler, so a GPU
process never pays for, or races on, a rebuild.
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


def build(verbose: bool = False) -> ModuleType:
    """Compile every CUDA source for sm_100a into ``csrc/_build`` and import it."""

    global _module
    os.makedirs(BUILD_DIR, exist_ok=True)
    from torch.utils.cpp_extension import load

    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    mod = load(
        name=MODULE_NAME,
        sources=sources(),
        build_directory=BUILD_DIR,
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=list(CUDA_FLAGS),
        extra_include_paths=[CSRC_DIR],
        extra_ldflags=[],
        verbose=verbose,
    )
    _module = mod
    return mod


def load() -> ModuleType:
    """Import the prebuilt library; raise ImportError if it has not been built."""

    global _module
    if _module is not None:
        return _module
    if MODULE_NAME in sys.modules:
        _module = sys.modules[MODULE_NAME]
        return _module
    if not os.path.exists(SO_PATH):
        raise ImportError(
            f"koochak_b200 native library not built ({SO_PATH} missing); "
            "run `python -c 'import __graft_entry__ as g; g.build()'` or koochak_b200._native_build.build()"
        )
    import torch  # noqa: F401  (the extension links against torch's libraries)

    spec = importlib.util.spec_from_file_location(MODULE_NAME, SO_PATH)
    assert spec is not None and spec.loader is not None
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[MODULE_NAME] = mod
    _module = mod
    return mod


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(SO_PATH)
