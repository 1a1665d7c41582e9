"""MoE-LoRA layers with the reference's interface, running on the sm_100a kernels.

Same classes and signatures as stageml/moe_lora_layers.py of the reference:

  DynamicMoELoRALayer(expert_weight, adapters, expert_bias=None)
      .forward(x, expert_ids, routing_weights, adapter_ids)
      out[t] = sum_k w[t,k] * (x_t W[e]^T + b[e] + s_a (x_t A_a[e]^T) B_a[e]^T)
      (stageml/moe_lora_layers.py:63-90)
  MaterializedMoELoRALayer(expert_weight, adapters, expert_bias=None)
      the stage-0 fold W[e] + s_a B_a[e] A_a[e] for every (adapter, expert) at
      construction (:104-110), then routed GEMMs on the merged weights (:117-142)

The per-token Python loops of the reference become one call of the routed
grouped GEMM (stageml_b200.ops.moe_linear): a stable (expert, tenant)
permutation, the gather + LoRA shrink, the tcgen05 grouped GEMM with the LoRA
expand on the tensor cores and the routing weight in its epilogue, and the
combine. Adapters are packed into zero-padded banks once at construction.
Inputs must be CUDA bf16/fp16 tensors; there is no CPU fallback.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn as nn

from ._packing import pack_lora_bank, pad_dim, pad_last, padded_rank, require_16bit, require_cuda, round_up


@dataclass
class MoEAdapterSpec:
    name: str
    A: torch.Tensor  # [E, r, in]
    B: torch.Tensor  # [E, out, r]
    scaling: float

    def __post_init__(self) -> None:
        if self.A.ndim != 3:
            raise ValueError("A must have shape num_experts by rank by in_features")
        if self.B.ndim != 3:
            raise ValueError("B must have shape num_experts by out_features by rank")
        if self.A.shape[0] != self.B.shape[0]:
            raise ValueError("A and B must have the same number of experts")
        if self.A.shape[1] != self.B.shape[2]:
            raise ValueError("A rank must match B rank")

    @property
    def num_experts(self) -> int:
        return int(self.A.shape[0])

    @property
    def rank(self) -> int:
        return int(self.A.shape[1])

    @property
    def in_features(self) -> int:
        return int(self.A.shape[2])

    @property
    def out_features(self) -> int:
        return int(self.B.shape[1])


def _check_routing(x, expert_ids, routing_weights, adapter_ids) -> None:
    if expert_ids.ndim != 2:
        raise ValueError("expert_ids must have shape tokens by top_k")
    if routing_weights.shape != expert_ids.shape:
        raise ValueError("routing_weights must match expert_ids")
    if x.shape[0] != expert_ids.shape[0] or x.shape[0] != len(adapter_ids):
        raise ValueError("token dimension mismatch")


class _MoELinearBase(nn.Module):
    def _setup(self, expert_weight: torch.Tensor, expert_bias: torch.Tensor | None) -> None:
        if expert_weight.ndim != 3:
            raise ValueError("expert_weight must have shape num_experts by out_features by in_features")
        self.num_experts, self.out_features, self.in_features = (int(s) for s in expert_weight.shape)
        self.k_pad = round_up(self.in_features, 8)
        self.n_pad = round_up(self.out_features, 8)
        if expert_bias is not None:
            self.register_buffer("expert_bias", pad_last(expert_bias.detach().clone(), self.n_pad).contiguous())
        else:
            self.expert_bias = None

    def _pad_x(self, x: torch.Tensor) -> torch.Tensor:
        return pad_last(x, self.k_pad).contiguous()

    def _adapter_index_tensor(self, adapter_ids: Sequence, device) -> torch.Tensor:
        return torch.tensor([self._adapter_index(a) for a in adapter_ids], dtype=torch.int32, device=device)


class DynamicMoELoRALayer(_MoELinearBase):
    """Per-token adapter LoRA on a routed expert linear, computed on the fly."""

    def __init__(self, expert_weight: torch.Tensor, adapters: Sequence[MoEAdapterSpec],
                 expert_bias: torch.Tensor | None = None):
        super().__init__()
        self._setup(expert_weight, expert_bias)
        w = pad_dim(pad_last(expert_weight.detach(), self.k_pad), 1, self.n_pad)
        self.register_buffer("expert_weight", w.contiguous())
        self.adapters = {a.name: a for a in adapters}
        self.adapter_names = list(self.adapters.keys())
        self.name_to_index = {n: i for i, n in enumerate(self.adapter_names)}
        specs = [self.adapters[n] for n in self.adapter_names]
        self.rank_pad = padded_rank(max((a.rank for a in specs), default=0))
        if specs:
            a_bank, b_bank = pack_lora_bank([a.A for a in specs], [a.B for a in specs], self.k_pad, self.n_pad,
                                            self.rank_pad, w.dtype, w.device)
            self.register_buffer("lora_a", a_bank)  # [n, E, r_pad, K]
            self.register_buffer("lora_b", b_bank)  # [n, E, N, r_pad]
        else:
            self.lora_a = self.lora_b = None
        self.register_buffer("lora_scale", torch.tensor([float(a.scaling) for a in specs], dtype=torch.float32,
                                                        device=w.device))

    def _adapter_name(self, adapter_id) -> str:
        if isinstance(adapter_id, int):
            return self.adapter_names[adapter_id]
        return str(adapter_id)

    def _adapter_index(self, adapter_id) -> int:
        return self.name_to_index[self._adapter_name(adapter_id)]

    def forward(self, x, expert_ids, routing_weights, adapter_ids):
        _check_routing(x, expert_ids, routing_weights, adapter_ids)
        require_cuda(x, "DynamicMoELoRALayer")
        require_16bit(x, "DynamicMoELoRALayer")
        from . import ops

        ten = self._adapter_index_tensor(adapter_ids, x.device)
        y = ops.moe_linear(self._pad_x(x), self.expert_weight, expert_ids.contiguous(),
                           routing_weights.to(torch.float32).contiguous(), bias=self.expert_bias, tenant_ids=ten,
                           n_experts=self.num_experts, n_tenants=len(self.adapter_names), rank=self.rank_pad,
                           lora_a=self.lora_a, lora_b=self.lora_b, lora_scale=self.lora_scale)
        return y[:, : self.out_features]


class MaterializedMoELoRALayer(_MoELinearBase):
    """Stage-0 folded W[e] + s_a B_a[e] A_a[e] for every (adapter, expert); routed GEMMs at run time."""

    def __init__(self, expert_weight: torch.Tensor, adapters: Sequence[MoEAdapterSpec],
                 expert_bias: torch.Tensor | None = None):
        super().__init__()
        self._setup(expert_weight, expert_bias)
        self.adapter_names = [a.name for a in adapters]
        self.name_to_index = {n: i for i, n in enumerate(self.adapter_names)}
        w = pad_dim(pad_last(expert_weight.detach(), self.k_pad), 1, self.n_pad).contiguous()
        merged = []
        for a in adapters:
            if a.num_experts != expert_weight.shape[0]:
                raise ValueError("adapter and expert weights disagree on expert count")
            merged.append(self._fold(w, a))
        if merged:
            self.register_buffer("merged_weight", torch.stack(merged, 0).contiguous())  # [nA, E, N, K]
        else:
            self.register_buffer("merged_weight", w.new_zeros((0, *w.shape)))

    def _fold(self, w: torch.Tensor, a: MoEAdapterSpec) -> torch.Tensor:
        from . import ops

        require_cuda(w, "MaterializedMoELoRALayer")
        A = pad_last(a.A.detach().to(w.dtype), self.k_pad).contiguous()            # [E, r, K]
        B = pad_dim(a.B.detach().to(w.dtype), 1, self.n_pad).contiguous()          # [E, N, r]
        scale = torch.full((w.shape[0],), float(a.scaling), dtype=torch.float32, device=w.device)
        return ops.lora_fold(w, A, B, scale, layout=0)  # W[e] + s * B[e] @ A[e]

    def _adapter_index(self, adapter_id) -> int:
        if isinstance(adapter_id, int):
            return int(adapter_id)
        return self.name_to_index[str(adapter_id)]

    def forward(self, x, expert_ids, routing_weights, adapter_ids):
        _check_routing(x, expert_ids, routing_weights, adapter_ids)
        require_cuda(x, "MaterializedMoELoRALayer")
        require_16bit(x, "MaterializedMoELoRALayer")
        from . import ops

        ten = self._adapter_index_tensor(adapter_ids, x.device)
        nA, E = self.merged_weight.shape[0], self.merged_weight.shape[1]
        y = ops.moe_linear(self._pad_x(x), self.merged_weight.view(nA * E, self.n_pad, self.k_pad),
                           expert_ids.contiguous(), routing_weights.to(torch.float32).contiguous(),
                           bias=self.expert_bias, tenant_ids=ten, n_experts=E, group_by_tenant=True, n_tenants=nA)
        return y[:, : self.out_features]


class NonMaterializingFusedMoELoRAReference(DynamicMoELoRALayer):
    pass


def make_random_moe_adapters(*, num_adapters: int, num_experts: int, in_features: int, out_features: int,
                             ranks: int | Sequence[int], dtype: torch.dtype, device: torch.device,
                             scaling: float | None = None) -> list[MoEAdapterSpec]:
    """Random adapters, A ~ N(0, 1/in), B ~ N(0, 1/rank), scaling 16/rank unless given
    (stageml/moe_lora_layers.py:149-171)."""
    if isinstance(ranks, int):
        rank_values = [int(ranks)] * num_adapters
    else:
        seq = list(ranks)
        rank_values = [int(seq[i % len(seq)]) for i in range(num_adapters)]
    out = []
    for i, r in enumerate(rank_values):
        s = float(scaling if scaling is not None else 16.0 / float(r))
        A = torch.randn(num_experts, r, in_features, device=device, dtype=dtype) / (in_features ** 0.5)
        B = torch.randn(num_experts, out_features, r, device=device, dtype=dtype) / (r ** 0.5)
        out.append(MoEAdapterSpec(name=f"adapter_{i}", A=A, B=B, scaling=s))
    return out


def make_round_robin_adapter_ids(num_tokens: int, num_adapters: int) -> list[str]:
    return [f"adapter_{i % num_adapters}" for i in range(num_tokens)]


def normalize_routing_weights(expert_ids: torch.Tensor, weights: torch.Tensor | None = None) -> torch.Tensor:
    """weights / max(sum(weights), 1e-12) per token in fp32 (stageml/moe_lora_layers.py:178-183)."""
    if weights is None:
        weights = torch.ones_like(expert_ids, dtype=torch.float32)
    weights = weights.to(torch.float32)
    return weights / weights.sum(dim=1, keepdim=True).clamp_min(1e-12)


__all__ = ["MoEAdapterSpec", "DynamicMoELoRALayer", "MaterializedMoELoRALayer",
           "NonMaterializingFusedMoELoRAReference", "make_random_moe_adapters", "make_round_robin_adapter_ids",
           "normalize_routing_weights"]
