"""Loading of the native libraries built in ``stageml_b200/lib``.

``load_torch_ops()`` registers the ``torch.ops.stageml`` namespace from
``libstageml_torch.so``; ``load_capi()`` opens ``libstageml_b200.so`` with ctypes
for direct C-ABI calls. Both fail loudly: there is no CPU or Python fallback
for the residual path, and a missing library is an error, never a silent
switch to another implementation.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIBDIR = Path(__file__).resolve().parent / "lib"
CORE_LIB = LIBDIR / "libstageml_b200.so"
TORCH_LIB = LIBDIR / "libstageml_torch.so"

_lock = threading.Lock()
_torch_loaded = False
_capi = None


class NativeLibraryMissing(RuntimeError):
    """The CUDA extension of stageml_b200 is not built or cannot be loaded."""


def _need(path: Path) -> None:
    if not path.exists():
        raise NativeLibraryMissing(
            f"{path.name} not found in {path.parent}; build it with `python -m stageml_b200.build` "
            "(the StageML B200 residual path has no CPU fallback)"
        )


def load_torch_ops() -> None:
    """Register ``torch.ops.stageml.*`` (idempotent)."""
    global _torch_loaded
    if _torch_loaded:
        return
    with _lock:
        if _torch_loaded:
            return
        import torch

        _need(CORE_LIB)
        _need(TORCH_LIB)
        # load the core library first so the op library's $ORIGIN dependency resolves to this copy
        ctypes.CDLL(str(CORE_LIB), mode=ctypes.RTLD_GLOBAL)
        torch.ops.load_library(str(TORCH_LIB))
        _torch_loaded = True


def torch_ops_path() -> str:
    """Path of the op library, the value to put in ``STAGEML_CUSTOM_OP_LIB``."""
    return str(TORCH_LIB)


def load_capi() -> ctypes.CDLL:
    """Open ``libstageml_b200.so`` and declare the C ABI signatures."""
    global _capi
    if _capi is not None:
        return _capi
    with _lock:
        if _capi is None:
            _need(CORE_LIB)
            lib = ctypes.CDLL(str(CORE_LIB), mode=ctypes.RTLD_GLOBAL)
            from . import capi as _decl

            _decl.declare(lib)
            _capi = lib
    return _capi


def native_loaded_paths() -> list[str]:
    """Native libraries of this package mapped into the current process."""
    out = []
    try:
        with open("/proc/self/maps") as fh:
            for line in fh:
                p = line.strip().split()[-1]
                if p.startswith(str(LIBDIR)) and p not in out:
                    out.append(p)
    except OSError:
        pass
    return out


def ensure_cuda_device(t) -> None:
    if not getattr(t, "is_cuda", False):
        raise RuntimeError(
            "stageml_b200 runs on CUDA tensors only (sm_100a); got a tensor on "
            f"{getattr(t, 'device', '?')}. There is no CPU fallback."
        )


__all__ = [
    "NativeLibraryMissing",
    "load_torch_ops",
    "load_capi",
    "torch_ops_path",
    "native_loaded_paths",
    "ensure_cuda_device",
    "CORE_LIB",
    "TORCH_LIB",
]

if os.environ.get("STAGEML_B200_EAGER_LOAD") == "1":  # pragma: no cover
    load_torch_ops()
