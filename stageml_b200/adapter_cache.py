"""Cost-based adapter residual cache with the reference's interface (stageml/adapter_cache.py).

  StageMLCostBasedAdapterCache(weight, adapters, *, cached_adapter_names, bias=None)
      hot adapters folded once at stage 0, W_i = W + s_i B_i A_i (:72-81); cold
      adapters stay dynamic, y = x W^T + s_i (x A_i^T) B_i^T (:83-100)
  choose_hot_adapters(request_counts, adapters, *, in_features, out_features, dtype, memory_budget_mb)
      cache the most requested adapters until the byte budget is spent (:106-140)

A forward is one grouped tcgen05 GEMM (stageml_b200.ops.lora_linear) over the
weight bank [W, W_cached...]: rows of cached adapters select their folded
weight, rows of dynamic adapters select W plus a tensor-core LoRA expand.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Mapping, Sequence

import torch

from .adapter_bank import AdapterSpec, _DenseBase


@dataclass(frozen=True)
class AdapterCacheDecision:
    """Decision for one adapter in the cache policy."""

    name: str
    cached: bool
    estimated_bytes: int
    use_count: int


class StageMLCostBasedAdapterCache(_DenseBase):
    """Mixed cached / dynamic LoRA layer."""

    def __init__(self, weight: torch.Tensor, adapters: Sequence[AdapterSpec], *, cached_adapter_names: Sequence[str],
                 bias: torch.Tensor | None = None):
        super().__init__()
        w = self._setup(weight, bias)
        self.register_buffer("weight", w)
        self._pack_adapters(adapters, w)
        self.cached_adapter_names = list(cached_adapter_names)
        self.cached_name_to_index = {n: i for i, n in enumerate(self.cached_adapter_names)}
        if self.cached_adapter_names:
            folded = self._fold(w, [self.adapters[n] for n in self.cached_adapter_names])
            bank = torch.cat([w[None], folded], 0)
        else:
            bank = w[None]
        self.register_buffer("weight_bank", bank.contiguous())  # [1 + n_cached, N, K]

    @property
    def cached_merged_weights(self) -> torch.Tensor:
        return self.weight_bank[1:, : self.out_features, : self.in_features]

    def forward(self, x: torch.Tensor, adapter_ids: Sequence[str]) -> torch.Tensor:
        from . import ops

        xp = self._prep(x, adapter_ids)
        grp, ten = [], []
        for name in adapter_ids:
            ci = self.cached_name_to_index.get(name)
            if ci is None:
                grp.append(0)
                ten.append(self.adapter_index[name])
            else:
                grp.append(ci + 1)
                ten.append(-1)
        grp_t = torch.tensor(grp, dtype=torch.int32, device=x.device)
        ten_t = torch.tensor(ten, dtype=torch.int32, device=x.device)
        y = ops.lora_linear(xp, self.weight_bank, bias=self.bias, row_group=grp_t if len(self.cached_adapter_names)
                            else None, row_tenant=ten_t, n_tenants=len(self.adapter_order), rank=self.rank_pad,
                            lora_a=self.lora_a, lora_b=self.lora_b, lora_scale=self.lora_scale)
        return y[:, : self.out_features]

    def cached_memory_bytes(self) -> int:
        return int(len(self.cached_adapter_names) * self.out_features * self.in_features * self.weight.element_size())


def choose_hot_adapters(request_counts: Mapping[str, int], adapters: Sequence[AdapterSpec], *, in_features: int,
                        out_features: int, dtype: torch.dtype,
                        memory_budget_mb: float) -> tuple[list[str], list[AdapterCacheDecision]]:
    """Cache adapters by descending request count (ties by name) while the folded weights fit the budget."""
    per_adapter = int(in_features * out_features * torch.empty((), dtype=dtype).element_size())
    budget = int(memory_budget_mb * 1024 * 1024)
    ranked = sorted((a.name for a in adapters), key=lambda n: (-int(request_counts.get(n, 0)), n))
    cached: list[str] = []
    used = 0
    decisions: list[AdapterCacheDecision] = []
    for name in ranked:
        count = int(request_counts.get(name, 0))
        take = used + per_adapter <= budget and count > 0
        if take:
            cached.append(name)
            used += per_adapter
        decisions.append(AdapterCacheDecision(name=name, cached=take, estimated_bytes=per_adapter, use_count=count))
    return cached, decisions


__all__ = ["AdapterCacheDecision", "StageMLCostBasedAdapterCache", "choose_hot_adapters"]
