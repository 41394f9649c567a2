"""Builds and loads the package's native extensions in-tree.

Two extensions:
- ``atlas_host``: pure C++ (page pool, route views, tree dedup) -- needed on CPU too;
- ``atlas_cuda``: the sm_100a kernels (tcgen05/TMA GEMM, paged attention,
  fused norm/rope/append, KV copy, top-k, collectives).

Both are compiled with ``torch.utils.cpp_extension.load`` into
``ops/_ext/<name>/`` inside the package so the shared objects ship with the
source tree.  CUDA code is compiled only for ``sm_100a``.
"""

from __future__ import annotations

import os
import threading
from pathlib import Path

import torch  # noqa: F401  (libtorch is loaded before the extension modules that link to it)

_PKG = Path(__file__).resolve().parent.parent
_CSRC = _PKG / "csrc"
_EXT_ROOT = Path(__file__).resolve().parent / "_ext"
_LOCK = threading.Lock()
_CACHE: dict[str, object] = {}

CUDA_ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _load(name: str, sources: list[Path], *, cuda: bool, verbose: bool = False):
    with _LOCK:
        if name in _CACHE:
            return _CACHE[name]
        from torch.utils.cpp_extension import load

        build_dir = _EXT_ROOT / name
        build_dir.mkdir(parents=True, exist_ok=True)
        kwargs: dict = dict(
            name=name,
            sources=[str(s) for s in sources],
            build_directory=str(build_dir),
            extra_cflags=["-O3", "-std=c++17"],
            verbose=verbose or bool(os.environ.get("ATLAS_BUILD_VERBOSE")),
        )
        if cuda:
            kwargs["extra_cuda_cflags"] = [
                *CUDA_ARCH_FLAGS,
                "-O3",
                "-lineinfo",
                "-std=c++17",
                "--expt-relaxed-constexpr",
                "-U__CUDA_NO_HALF_OPERATORS__",
                "-U__CUDA_NO_HALF_CONVERSIONS__",
                "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
                f"-I{_CSRC / 'cuda'}",
            ]
            kwargs["extra_include_paths"] = [str(_CSRC / "cuda")]
            kwargs["extra_ldflags"] = ["-lcuda"]
        mod = load(**kwargs)
        _CACHE[name] = mod
        return mod


def host():
    """The C++ host extension (always available; builds on first use)."""
    return _load("atlas_host", [_CSRC / "host" / "page_pool.cpp"], cuda=False)


CUDA_SOURCES = [
    "bindings.cpp",
    "gemm_tcgen05.cu",
    "attention.cu",
    "elementwise.cu",
    "kvcache.cu",
    "sampling.cu",
    "topk_noalloc.cu",
    "tp.cu",
    "peer_ring.cu",
    "gemm_fp8.cu",
]


def cuda():
    """The sm_100a kernel extension.  Raises if it cannot be built or loaded."""
    return _load("atlas_cuda", [_CSRC / "cuda" / s for s in CUDA_SOURCES], cuda=True)
