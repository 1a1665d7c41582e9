"""Python entry points of the B200 residual path.

Thin functions over ``torch.ops.stageml.*`` (csrc/torch_ops.cpp -> C ABI ->
sm_100a kernels). Each one takes CUDA tensors and launches on the current
stream. Fake (meta) implementations are registered so the ops trace under
``torch.compile`` / FakeTensor without running.
"""

from __future__ import annotations

from typing import Optional

import torch

from ._native import ensure_cuda_device, load_torch_ops

load_torch_ops()
_ops = torch.ops.stageml


def _register_fakes() -> None:
    lib = torch.library

    @lib.register_fake("stageml::residual_moe")
    def _(hidden, gate_up, down, topk_weights, topk_ids):
        return hidden.new_empty((hidden.shape[0], down.shape[1]))

    @lib.register_fake("stageml::moe_forward")
    def _(x, gate_up, down, topk_weights, topk_ids, router_w, k, n_shared, renormalize, tenant_ids, n_tenants, rank,
          lora_a13, lora_b13, lora_a2, lora_b2, lora_scale, gate_up_scale, down_scale, T_dev=None, fold_slot=None,
          n_fold=0, down_group=None):
        return x.new_empty((x.shape[0], x.shape[1]))

    @lib.register_fake("stageml::route_topk")
    def _(x, gate_w, k, renormalize):
        T = x.shape[0]
        return (x.new_empty((T, k), dtype=torch.int32), x.new_empty((T, k), dtype=torch.float32),
                x.new_empty((T, gate_w.shape[0]), dtype=torch.float32))

    @lib.register_fake("stageml::topk_from_logits")
    def _(logits, k, renormalize):
        T = logits.shape[0]
        return logits.new_empty((T, k), dtype=torch.int32), logits.new_empty((T, k), dtype=torch.float32)

    @lib.register_fake("stageml::lora_fold")
    def _(W, A, B, scale, layout):
        if A.dim() == 3:
            return W.new_empty((A.shape[0], W.shape[-2], W.shape[-1]))
        return W.new_empty(W.shape)

    @lib.register_fake("stageml::lora_linear")
    def _(x, w_bank, bias, row_group, row_tenant, n_tenants, rank, lora_a, lora_b, lora_scale):
        return x.new_empty((x.shape[0], w_bank.shape[1]))

    @lib.register_fake("stageml::moe_linear")
    def _(x, weight, bias, topk_ids, topk_weights, tenant_ids, n_experts, group_by_tenant, n_tenants, rank, lora_a,
          lora_b, lora_scale):
        return x.new_empty((x.shape[0], weight.shape[1]))

    @lib.register_fake("stageml::combine_rows")
    def _(y, pair_row, T, kk):
        return y.new_empty((T, y.shape[1]))

    @lib.register_fake("stageml::lora_gemv_f32")
    def _(x, W, A, B, scale):
        return x.new_empty((x.shape[0], W.shape[1]))


try:
    _register_fakes()
except Exception:  # pragma: no cover - re-registration in the same process
    pass


def residual_moe(hidden, gate_up, down, topk_weights, topk_ids):
    """The reference's ``stageml::residual_moe`` (csrc/stageml_residual_op.cpp:17-19), semantics of
    ``_fallback_moe`` (stageml/custom_op_registry.py:23-37)."""
    ensure_cuda_device(hidden)
    return _ops.residual_moe(hidden, gate_up.contiguous(), down.contiguous(), topk_weights.contiguous(),
                             topk_ids.contiguous())


def moe_forward(x, gate_up, down, *, topk_weights=None, topk_ids=None, router_w=None, k: int = 2, n_shared: int = 0,
                renormalize: bool = True, tenant_ids=None, n_tenants: int = 0, rank: int = 0, lora_a13=None,
                lora_b13=None, lora_a2=None, lora_b2=None, lora_scale=None, gate_up_scale=None, down_scale=None,
                T_dev=None, fold_slot=None, n_fold: int = 0, down_group=None):
    """One MoE-LoRA FFN layer (router -> permutation -> SwiGLU experts with per-tenant LoRA -> combine).

    T_dev: optional CUDA int32 tensor; only the first T_dev[0] tokens are valid (the rest are skipped and
    their output rows are left unwritten), for token counts known only on the device.
    fold_slot: optional CUDA int32 [n_tenants, E_tot]; entry (a, e) = s >= 0 runs tenant a's pairs of
    expert e on folded weight set s, stored as group E_tot + s of gate_up / down ([E_tot + n_fold, ...]),
    without dynamic LoRA; -1 = base weights plus the tenant's LoRA. One permutation, one set of GEMMs.
    down_group: optional CUDA int32 [E_tot + n_fold] with entries in [0, E_tot): weight group g takes
    down[down_group[g]] (down then holds the E_tot base experts), for folded sets whose adapters leave
    w2 unchanged.
    """
    ensure_cuda_device(x)
    if topk_ids is not None:
        k = int(topk_ids.shape[1])
    return _ops.moe_forward(x, gate_up, down, topk_weights, topk_ids, router_w, int(k), int(n_shared),
                            bool(renormalize), tenant_ids, int(n_tenants), int(rank), lora_a13, lora_b13, lora_a2,
                            lora_b2, lora_scale, gate_up_scale, down_scale, T_dev, fold_slot, int(n_fold),
                            down_group)


def route_topk(x, gate_w, k: int, renormalize: bool = True):
    """Router logits (fp32), softmax, top-k, renormalisation -> (ids int32, weights fp32, logits fp32)."""
    ensure_cuda_device(x)
    return _ops.route_topk(x, gate_w, int(k), bool(renormalize))


def topk_from_logits(logits, k: int, renormalize: bool = True):
    ensure_cuda_device(logits)
    return _ops.topk_from_logits(logits, int(k), bool(renormalize))


PLAN_FIELDS = ("row_token", "row_tenant", "row_weight", "row_pair", "pair_row", "tile_group", "group_offsets",
               "group_counts", "num_tiles")


def permute(ids, weights=None, tenant_ids=None, *, n_experts_total: int, n_shared: int = 0, n_tenants: int = 0,
            group_by_tenant: bool = False) -> dict:
    """Stable (expert, tenant) permutation with 128-row padded expert segments; returns the plan arrays."""
    ensure_cuda_device(ids)
    out = _ops.permute(ids, weights, tenant_ids, int(n_experts_total), int(n_shared), int(n_tenants),
                       bool(group_by_tenant))
    return dict(zip(PLAN_FIELDS, out))


def lora_fold(W, A, B, scale, layout: int = 0):
    """W' = W + s * B @ A (layout 0, [out,in]) or W + s * A @ B (layout 1, [in,out]); batched over A/B."""
    ensure_cuda_device(W)
    if not torch.is_tensor(scale):
        n = A.shape[0] if A.dim() == 3 else 1
        scale = torch.full((n,), float(scale), dtype=torch.float32, device=W.device)
    return _ops.lora_fold(W.contiguous(), A.contiguous(), B.contiguous(), scale.to(torch.float32).contiguous(),
                          int(layout))


def lora_linear(x, w_bank, *, bias=None, row_group=None, row_tenant=None, n_tenants: int = 0, rank: int = 0,
                lora_a=None, lora_b=None, lora_scale=None):
    """Mixed-adapter dense linear: folded weights by row group, dynamic LoRA by row tenant."""
    ensure_cuda_device(x)
    return _ops.lora_linear(x, w_bank, bias, row_group, row_tenant, int(n_tenants), int(rank), lora_a, lora_b,
                            lora_scale)


def moe_linear(x, weight, topk_ids, topk_weights, *, bias=None, tenant_ids=None, n_experts: int,
               group_by_tenant: bool = False, n_tenants: int = 0, rank: int = 0, lora_a=None, lora_b=None,
               lora_scale=None):
    """Routed single-linear MoE-LoRA layer (DynamicMoELoRALayer / MaterializedMoELoRALayer)."""
    ensure_cuda_device(x)
    return _ops.moe_linear(x, weight, bias, topk_ids, topk_weights, tenant_ids, int(n_experts), bool(group_by_tenant),
                           int(n_tenants), int(rank), lora_a, lora_b, lora_scale)


def lora_gemv_f32(x, W, A=None, B=None, scale: float = 1.0):
    """fp32 y = x W + s (x A) B with W [in,out] (A None: y = x W)."""
    ensure_cuda_device(x)
    return _ops.lora_gemv_f32(x, W, A, B, float(scale))


def quantize_e4m3_rows(w):
    """Per-output-channel e4m3 quantization -> (q float8_e4m3fn, scale fp32)."""
    ensure_cuda_device(w)
    return _ops.quantize_e4m3_rows(w.contiguous())


def combine_rows(y, pair_row, T: int, kk: int):
    """out[t] = sum_j y[pair_row[t*kk + j]] (rows < 0 skipped), fp32 sum, one rounding."""
    ensure_cuda_device(y)
    return _ops.combine_rows(y.contiguous(), pair_row.to(torch.int32).contiguous(), int(T), int(kk))


def take_status(like) -> int:
    """Synchronise and return (then clear) the device status word of like's device (0 = ok)."""
    return int(_ops.take_status(like))


__all__ = [
    "residual_moe",
    "moe_forward",
    "route_topk",
    "topk_from_logits",
    "permute",
    "lora_fold",
    "lora_linear",
    "moe_linear",
    "lora_gemv_f32",
    "quantize_e4m3_rows",
    "combine_rows",
    "take_status",
    "PLAN_FIELDS",
]
