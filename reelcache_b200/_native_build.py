"""Builds and loads the package's native extension (CUDA for sm_100a plus C++ host code).

``build()`` compiles every source under ``csrc/`` in-tree with ``nvcc -gencode
arch=compute_100a,code=sm_100a`` through ``torch.utils.cpp_extension`` (ninja, incremental) and
leaves ``_build/reelcache_b200_C.so`` beside the package, so a copy of the tree carries the built
library. ``load()`` imports that library without invoking the compiler.
"""

from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
import threading

NAME = "reelcache_b200_C"
PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PACKAGE_DIR, "csrc")
BUILD_DIR = os.path.join(PACKAGE_DIR, "_build")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("REELCACHE_PTXAS_VERBOSE") else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

_lock = threading.Lock()
_module = None


def sources():
    found = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    found += sorted(glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True))
    return found


def library_path():
    return os.path.join(BUILD_DIR, NAME + ".so")


def build(verbose: bool = False):
    """Compile the extension in-tree for sm_100a (works without a GPU) and return the module."""
    global _module
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.makedirs(BUILD_DIR, exist_ok=True)
    from torch.utils import cpp_extension

    with _lock:
        module = cpp_extension.load(
            name=NAME,
            sources=sources(),
            extra_cflags=CXX_FLAGS,
            extra_cuda_cflags=CUDA_FLAGS,
            extra_include_paths=[CSRC],
            build_directory=BUILD_DIR,
            verbose=verbose,
            with_cuda=True,
        )
        _module = module
    return module


def load():
    """Import the prebuilt extension (raises ImportError with the path when it is missing)."""
    global _module
    if _module is not None:
        return _module
    with _lock:
        if _module is not None:
            return _module
        if NAME in sys.modules:
            _module = sys.modules[NAME]
            return _module
        path = library_path()
        if not os.path.exists(path):
            raise ImportError(
                f"reelcache_b200 native extension not built: {path} is missing; run "
                "`python -c 'import __graft_entry__ as g; g.build()'` or reelcache_b200._native_build.build()"
            )
        import torch  # noqa: F401  (loads libtorch / libc10 the extension links against)

        loader = importlib.machinery.ExtensionFileLoader(NAME, path)
        spec = importlib.util.spec_from_file_location(NAME, path, loader=loader)
        module = importlib.util.module_from_spec(spec)
        loader.exec_module(module)
        sys.modules[NAME] = module
        _module = module
    return _module
