"""Build and load the sm_100a extension (`dtb_C`) in-tree.

The CUDA sources live in ``csrc/``; they are compiled for Blackwell only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/dtb_C*.so`` inside the
package, so the built library travels with a copy of the source tree.

``lib()`` imports the built library directly and never rebuilds silently: a
machine with a GPU but no built library gets a loud error instead of a slow
fallback.
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent
SRC_DIR = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
NAME = "dtb_C"

SOURCES = ["bindings.cpp", "gemm.cu", "layernorm.cu", "embed_xent.cu", "optim.cu", "attention.cu", "attention_tc.cu", "comm.cu",
           "vmm.cpp"]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("DTB_PTXAS_VERBOSE") else "-Xptxas=-O3",
]

_lock = threading.Lock()
_lib = None


def _shared_libstdcxx() -> list[str]:
    """Linker input that binds the extension to the libstdc++ this process runs on.

    A toolchain whose ``libstdc++.so`` link is missing silently links the static
    ``libstdc++.a`` into the extension.  That private copy then mixes with the
    process's shared libstdc++ (which already owns the iostream/locale objects), and
    the first error message that formats a number (``TORCH_CHECK(..., n)``) crashes
    with SIGSEGV instead of raising.  Naming the loaded ``libstdc++.so.6`` on the
    link line resolves every C++ runtime symbol against it; the static archive the
    driver appends afterwards then contributes nothing.
    """
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                path = line.split()[-1] if line.strip() else ""
                if os.path.basename(path).startswith("libstdc++.so") and os.path.exists(path):
                    return [path]
    except OSError:
        pass
    import ctypes.util
    name = ctypes.util.find_library("stdc++")
    return [f"-l:{name}"] if name else []


def build(verbose: bool = False):
    """Compile every CUDA source for sm_100a and return the loaded module."""
    from torch.utils import cpp_extension

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    mod = cpp_extension.load(
        name=NAME,
        sources=[str(SRC_DIR / s) for s in SOURCES],
        build_directory=str(BUILD_DIR),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=CUDA_FLAGS,
        extra_ldflags=_shared_libstdcxx(),
        verbose=verbose,
        with_cuda=True,
    )
    global _lib
    _lib = mod
    return mod


def built_path() -> str | None:
    hits = sorted(glob.glob(str(BUILD_DIR / f"{NAME}*.so")))
    return hits[0] if hits else None


def available() -> bool:
    return built_path() is not None


def lib():
    """The loaded extension module.  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = built_path()
        if path is None:
            raise RuntimeError(
                f"the sm_100a extension is not built (expected {BUILD_DIR}/{NAME}.so); "
                "run `python -c 'import __graft_entry__ as g; g.build()'` from the repository root")
        import torch  # noqa: F401  (the extension links against libtorch)

        spec = importlib.util.spec_from_file_location(NAME, path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules[NAME] = mod
        _lib = mod
        return mod
