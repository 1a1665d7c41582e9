"""The C ABI library loads, exports exactly what include/stageml_b200.h declares, and its
host-side argument checks reject bad calls before any GPU work (no GPU needed)."""

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT
from stageml_b200 import capi
from stageml_b200._native import CORE_LIB, load_capi

HEADER = ROOT / "include" / "stageml_b200.h"


def declared_functions() -> set:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(stageml_[a-z0-9_]+)\s*\(", text))


def test_library_exports_exactly_the_header():
    out = subprocess.run(["nm", "-D", "--defined-only", str(CORE_LIB)], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    assert exported == declared_functions()


def test_ctypes_mirror_covers_every_function_and_struct():
    lib = load_capi()
    assert set(capi.SIGNATURES) == declared_functions()
    for which, S in capi.STRUCTS.items():
        assert ctypes.sizeof(S) == lib.stageml_struct_size(which), S.__name__
    assert lib.stageml_abi_version() >= 1


def test_plan_rows_cap():
    lib = load_capi()
    assert lib.stageml_plan_rows_cap(4096, 8) == 5120
    assert lib.stageml_plan_rows_cap(0, 8) == 128
    assert lib.stageml_plan_rows_cap(3, 64) == 384  # at most one padded segment per pair


@pytest.mark.parametrize("call", [
    lambda L: L.stageml_lora_fold(None, None, None, None, 1, 4, 4, 2, 0, 0, 0, 0, capi.BF16, None, None),
    lambda L: L.stageml_lora_fold(1, 1, 1, 1, 1, 4, 4, 2, 7, 0, 0, 0, capi.BF16, 1, None),
    lambda L: L.stageml_topk_from_logits(1, 4, 300, 2, 1, 1, 1, None),
    lambda L: L.stageml_topk_from_logits(1, 4, 8, 9, 1, 1, 1, None),
    lambda L: L.stageml_lora_gemv_f32(1, 1, None, None, 1.0, 17, 64, 64, 0, 1, 1, 1 << 20, None),
])
def test_invalid_arguments_are_rejected_on_the_host(call):
    lib = load_capi()
    rc = call(lib)
    assert rc == capi.ERR_INVALID_ARG
    assert lib.stageml_last_error().decode()


def test_moe_args_validation_and_workspace_query():
    lib = load_capi()
    a = capi.MoeArgs(T=0, H=4096, I=14336, E=8, k=2, act_dtype=capi.BF16, weight_dtype=capi.BF16, topk_ids=1,
                     ids_dtype=capi.I32)
    assert lib.stageml_moe_workspace_bytes(ctypes.byref(a)) > 0
    a.T = 2048
    need = lib.stageml_moe_workspace_bytes(ctypes.byref(a))
    assert need > 2048 * 2 * 14336 * 2  # holds the SwiGLU intermediate of the padded rows
    a.rank = 12  # ranks are 8, 16 or 32 after zero padding
    assert lib.stageml_moe_workspace_bytes(ctypes.byref(a)) == 0
    a.rank = 8
    assert lib.stageml_moe_workspace_bytes(ctypes.byref(a)) > 0
    a.rank = 16
    a.H = 4100  # not a multiple of 8
    assert lib.stageml_moe_forward(ctypes.byref(a), None, 0, None) == capi.ERR_INVALID_ARG
    a.H = 4096
    assert lib.stageml_moe_forward(ctypes.byref(a), None, 0, None) == capi.ERR_INVALID_ARG  # null tensors
    a2 = capi.MoeArgs(T=16, H=64, I=64, E=2, k=1, act_dtype=capi.BF16, weight_dtype=capi.E4M3, topk_ids=1,
                      ids_dtype=capi.I32, x=16, gate_up=16, down=16, out=16)
    # e4m3 weights need their per-row scales, and H, I multiples of 16
    assert lib.stageml_moe_forward(ctypes.byref(a2), None, 0, None) == capi.ERR_INVALID_ARG
    assert "scale" in lib.stageml_last_error().decode()
    a2.gate_up_scale = a2.down_scale = 16
    assert lib.stageml_moe_workspace_bytes(ctypes.byref(a2)) > 0
    assert lib.stageml_moe_forward(ctypes.byref(a2), None, 0, None) == capi.ERR_WORKSPACE
    a2.I = 72
    assert lib.stageml_moe_workspace_bytes(ctypes.byref(a2)) == 0


def test_workspace_too_small_is_reported():
    lib = load_capi()
    need = lib.stageml_residual_moe_workspace_bytes(64, 128, 128, 4, 2)
    assert need > 0
    rc = lib.stageml_residual_moe(16, 16, 16, 16, capi.F32, 16, capi.I64, 64, 128, 128, 4, 2, capi.BF16, 16, None,
                                  16, need - 1, None)
    assert rc == capi.ERR_WORKSPACE
