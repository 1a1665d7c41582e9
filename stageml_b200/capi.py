"""ctypes mirror of include/stageml_b200.h.

This is the binding a Python host (the reference's own language for this path)
would add to call the C ABI without torch's dispatcher: the structs mirror the
C layouts field for field (checked against ``stageml_struct_size``), and every
function gets explicit argtypes/restype.
"""

from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int32, c_int64, c_size_t, c_uint8, c_void_p

c_int32_p = POINTER(c_int32)
c_float_p = POINTER(c_float)

OK = 0
ERR_INVALID_ARG = 1
ERR_CUDA = 2
ERR_UNSUPPORTED = 3
ERR_WORKSPACE = 4

F32, BF16, F16, E4M3, I32, I64 = 0, 1, 2, 3, 4, 5
DEV_OK, DEV_TIMEOUT, DEV_PEER_TIMEOUT, DEV_BAD_INDEX = 0, 101, 105, 110


class MoePlan(ctypes.Structure):
    _fields_ = [
        ("row_token", c_void_p),
        ("row_tenant", c_void_p),
        ("row_weight", c_void_p),
        ("row_pair", c_void_p),
        ("pair_row", c_void_p),
        ("tile_group", c_void_p),
        ("group_offsets", c_void_p),
        ("group_counts", c_void_p),
        ("num_tiles", c_void_p),
        ("rows_cap", c_int64),
    ]


class MoeArgs(ctypes.Structure):
    _fields_ = [
        ("T", c_int),
        ("H", c_int),
        ("I", c_int),
        ("E", c_int),
        ("k", c_int),
        ("n_shared", c_int),
        ("act_dtype", c_int),
        ("weight_dtype", c_int),
        ("x", c_void_p),
        ("topk_ids", c_void_p),
        ("ids_dtype", c_int),
        ("topk_weights", c_void_p),
        ("weights_dtype", c_int),
        ("router_w", c_void_p),
        ("renormalize", c_int),
        ("tenant_ids", c_void_p),
        ("n_tenants", c_int),
        ("rank", c_int),
        ("gate_up", c_void_p),
        ("down", c_void_p),
        ("gate_up_scale", c_void_p),
        ("down_scale", c_void_p),
        ("lora_a13", c_void_p),
        ("lora_b13", c_void_p),
        ("lora_a2", c_void_p),
        ("lora_b2", c_void_p),
        ("lora_scale", c_void_p),
        ("out", c_void_p),
        ("status", c_void_p),
        ("plan_out", c_void_p),
        ("T_dev", c_void_p),
        ("fold_slot", c_void_p),
        ("n_fold", c_int),
        ("down_group", c_void_p),
    ]


class LoraLinearArgs(ctypes.Structure):
    _fields_ = [
        ("M", c_int),
        ("K", c_int),
        ("N", c_int),
        ("dtype", c_int),
        ("x", c_void_p),
        ("w_bank", c_void_p),
        ("n_groups", c_int),
        ("bias", c_void_p),
        ("row_group", c_void_p),
        ("row_tenant", c_void_p),
        ("n_tenants", c_int),
        ("rank", c_int),
        ("lora_a", c_void_p),
        ("lora_b", c_void_p),
        ("lora_scale", c_void_p),
        ("y", c_void_p),
        ("status", c_void_p),
    ]


class EpLayout(ctypes.Structure):
    _fields_ = [(n, c_size_t) for n in ("count_matrix", "flags_count", "flags_rows", "flags_return", "counters",
                                         "recv_tokens", "recv_expert", "recv_weight", "recv_tenant", "recv_source",
                                         "recv_x", "ret_y", "total")]


class EpArgs(ctypes.Structure):
    _fields_ = [
        ("world", c_int),
        ("rank", c_int),
        ("T", c_int),
        ("k", c_int),
        ("H", c_int),
        ("E_loc", c_int),
        ("act_dtype", c_int),
        ("epoch", c_int),
        ("tokens_cap", c_int64),
        ("timeout_ns", ctypes.c_uint64),
        ("peers", c_void_p),
        ("self", c_void_p),
        ("topk_ids", c_void_p),
        ("topk_weights", c_void_p),
        ("tenant_ids", c_void_p),
        ("x", c_void_p),
        ("pos", c_void_p),
        ("status", c_void_p),
    ]


# name -> (restype, argtypes)
SIGNATURES = {
    "stageml_last_error": (ctypes.c_char_p, []),
    "stageml_abi_version": (c_int, []),
    "stageml_struct_size": (c_size_t, [c_int]),
    "stageml_route_topk": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                   c_void_p, c_void_p]),
    "stageml_topk_from_logits": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "stageml_plan_rows_cap": (c_int64, [c_int64, c_int]),
    "stageml_permute_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "stageml_permute": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                POINTER(MoePlan), c_void_p, c_void_p, c_size_t, c_void_p]),
    "stageml_combine_rows": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "stageml_moe_workspace_bytes": (c_size_t, [POINTER(MoeArgs)]),
    "stageml_moe_forward": (c_int, [POINTER(MoeArgs), c_void_p, c_size_t, c_void_p]),
    "stageml_residual_moe_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "stageml_residual_moe": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int,
                                     c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "stageml_moe_linear_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int]),
    "stageml_moe_linear": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_int,
                                   c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                   c_int, c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "stageml_lora_fold": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int64,
                                  c_int64, c_int64, c_int, c_void_p, c_void_p]),
    "stageml_lora_linear_workspace_bytes": (c_size_t, [POINTER(LoraLinearArgs)]),
    "stageml_lora_linear": (c_int, [POINTER(LoraLinearArgs), c_void_p, c_size_t, c_void_p]),
    "stageml_lora_gemv_f32_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "stageml_lora_gemv_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int, c_int, c_int, c_int,
                                      c_void_p, c_void_p, c_size_t, c_void_p]),
    "stageml_lora_gemv_f32_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int, c_int, c_int,
                                              c_int, c_void_p, c_void_p]),
    "stageml_quantize_e4m3_rows": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p, c_void_p]),
    "stageml_stage_timer_enable": (c_int, [c_int]),
    "stageml_stage_timer_select": (c_int, [ctypes.c_uint]),
    "stageml_stage_timer_read": (c_int, [c_float_p, c_int32_p, c_int]),
    "stageml_launch_count": (ctypes.c_ulonglong, []),
    "stageml_ep_get_layout": (c_int, [c_int, c_int64, c_int, c_int, c_int, POINTER(EpLayout)]),
    "stageml_ep_workspace_alloc": (c_int, [c_size_t, POINTER(c_void_p), c_void_p]),
    "stageml_ep_workspace_free": (c_int, [c_void_p]),
    "stageml_ep_workspace_open": (c_int, [c_void_p, POINTER(c_void_p)]),
    "stageml_ep_workspace_close": (c_int, [c_void_p]),
    "stageml_ep_dispatch": (c_int, [POINTER(EpArgs), c_void_p]),
    "stageml_ep_return": (c_int, [POINTER(EpArgs), c_void_p, c_void_p]),
    "stageml_ep_combine": (c_int, [POINTER(EpArgs), c_void_p, c_void_p, c_void_p]),
}

STAGE_NAMES = ("route", "permute", "gather_shrink", "gemm_gate_up", "shrink_h", "gemm_down", "combine", "gemm",
               "fold", "gemv")

STRUCTS = {0: MoePlan, 1: MoeArgs, 2: LoraLinearArgs, 3: EpLayout, 4: EpArgs}


def declare(lib: ctypes.CDLL) -> None:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def check(lib: ctypes.CDLL, rc: int, what: str) -> None:
    if rc != OK:
        msg = lib.stageml_last_error()
        raise RuntimeError(f"{what} failed (code {rc}): {msg.decode() if msg else ''}")


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()


def stream_handle(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


__all__ = ["MoePlan", "MoeArgs", "LoraLinearArgs", "EpLayout", "EpArgs", "SIGNATURES", "STRUCTS", "declare", "check", "ptr",
           "stream_handle", "F32", "BF16", "F16", "E4M3", "I32", "I64", "OK"]
