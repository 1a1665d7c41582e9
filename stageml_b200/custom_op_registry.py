"""Registration of the ``stageml::residual_moe`` torch op (reference: stageml/custom_op_registry.py).

The reference declares the op in csrc/stageml_residual_op.cpp (a skeleton that
throws) and falls back to a per-token Python loop. Here the op library is the
built ``lib/libstageml_torch.so``: it registers ``residual_moe`` with the same
schema on the CUDA dispatch key only, backed by the sm_100a kernels.

  load_binary_custom_op()        load the library named by STAGEML_CUSTOM_OP_LIB (as the reference)
  register_native_custom_op()    load this package's op library
  ensure_stageml_custom_op(...)  make torch.ops.stageml.residual_moe callable

There is deliberately no Python or CPU fallback: ``allow_python_fallback`` is
accepted for signature compatibility and means "fall back to this package's
native library" when STAGEML_CUSTOM_OP_LIB is unset or fails to load.
"""

from __future__ import annotations

import os

import torch

from ._native import load_torch_ops, torch_ops_path


def load_binary_custom_op() -> bool:
    """Load the op library named by STAGEML_CUSTOM_OP_LIB, if set (stageml/custom_op_registry.py:40-48)."""
    lib = os.environ.get("STAGEML_CUSTOM_OP_LIB")
    if not lib:
        return False
    if os.path.realpath(lib) == os.path.realpath(torch_ops_path()):
        load_torch_ops()
    else:
        torch.ops.load_library(lib)
    return True


def register_native_custom_op() -> bool:
    """Register stageml::residual_moe from this package's native library."""
    load_torch_ops()
    return True


def _op_available() -> bool:
    try:
        getattr(torch.ops.stageml, "residual_moe")
        return True
    except (AttributeError, RuntimeError):
        return False


def ensure_stageml_custom_op(*, allow_python_fallback: bool = True) -> bool:
    """Ensure a callable torch.ops.stageml.residual_moe exists (stageml/custom_op_registry.py:78-94)."""
    try:
        load_binary_custom_op()
    except Exception:
        if not allow_python_fallback:
            raise
    if _op_available():
        return True
    if allow_python_fallback:
        return register_native_custom_op() and _op_available()
    return False


__all__ = ["load_binary_custom_op", "register_native_custom_op", "ensure_stageml_custom_op"]
