"""Multi-tenant dense LoRA layers with the reference's interface (stageml/adapter_bank.py).

  DynamicLoRALinear(weight, adapters, bias=None).forward(x, adapter_ids)
      y = x W^T + b + s_a (x A_a^T) B_a^T per row (stageml/adapter_bank.py:42-69)
  StageMLAdapterBankLinear(weight, adapters, bias=None).forward(x, adapter_ids)
      stage-0 fold W_a = W + s_a B_a A_a for every adapter (:90-94), rows grouped
      by adapter at run time (:101-109)
  OnTheFlyMergeLinear(weight, adapters, bias=None).forward(x, adapter_ids)
      the slow baseline that merges the present adapters on every call (:112-135)

Each forward is one call of the grouped tcgen05 GEMM (stageml_b200.ops.lora_linear):
rows select a weight group (base or folded) and, for dynamic rows, a LoRA tenant
whose expand runs on the tensor cores in the same accumulator. Inputs must be
CUDA bf16/fp16 tensors; there is no CPU fallback.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn as nn

from ._packing import pack_lora_bank, pad_dim, pad_last, padded_rank, require_16bit, require_cuda, round_up


@dataclass
class AdapterSpec:
    """One LoRA adapter for one linear projection."""

    name: str
    A: torch.Tensor  # [rank, in_features]
    B: torch.Tensor  # [out_features, rank]
    scaling: float


class _DenseBase(nn.Module):
    def _setup(self, weight: torch.Tensor, bias: torch.Tensor | None) -> None:
        self.out_features, self.in_features = (int(s) for s in weight.shape)
        self.k_pad = round_up(self.in_features, 8)
        self.n_pad = round_up(self.out_features, 8)
        w = pad_dim(pad_last(weight.detach(), self.k_pad), 0, self.n_pad).contiguous()
        if bias is not None:
            self.register_buffer("bias", pad_last(bias.detach().clone(), self.n_pad).contiguous())
        else:
            self.bias = None
        return w

    def _pack_adapters(self, adapters: Sequence[AdapterSpec], w: torch.Tensor) -> None:
        self.adapters = {a.name: a for a in adapters}
        self.adapter_order = [a.name for a in adapters]
        self.adapter_index = {n: i for i, n in enumerate(self.adapter_order)}
        self.rank_pad = padded_rank(max((int(a.A.shape[0]) for a in adapters), default=0))
        if adapters:
            a_bank, b_bank = pack_lora_bank([a.A for a in adapters], [a.B for a in adapters], self.k_pad, self.n_pad,
                                            self.rank_pad, w.dtype, w.device)
            self.register_buffer("lora_a", a_bank)  # [n, r_pad, K]
            self.register_buffer("lora_b", b_bank)  # [n, N, r_pad]
        else:
            self.lora_a = self.lora_b = None
        self.register_buffer("lora_scale", torch.tensor([float(a.scaling) for a in adapters], dtype=torch.float32,
                                                        device=w.device))

    def _fold(self, w: torch.Tensor, adapters: Sequence[AdapterSpec]) -> torch.Tensor:
        """[n, N, K] = W + s_a B_a A_a for each adapter (one batched fold launch)."""
        from . import ops

        require_cuda(w, type(self).__name__)
        r = padded_rank(max(int(a.A.shape[0]) for a in adapters))
        A, B = pack_lora_bank([a.A for a in adapters], [a.B for a in adapters], self.k_pad, self.n_pad, r, w.dtype,
                              w.device)
        scale = torch.tensor([float(a.scaling) for a in adapters], dtype=torch.float32, device=w.device)
        return ops.lora_fold(w, A, B, scale, layout=0)

    def _prep(self, x: torch.Tensor, adapter_ids: Sequence[str]) -> torch.Tensor:
        if x.shape[0] != len(adapter_ids):
            raise ValueError("batch dimension must match number of adapter ids")
        require_cuda(x, type(self).__name__)
        require_16bit(x, type(self).__name__)
        return pad_last(x, self.k_pad).contiguous()


class DynamicLoRALinear(_DenseBase):
    """Mixed-adapter LoRA layer that keeps A and B as separate factors."""

    def __init__(self, weight: torch.Tensor, adapters: Sequence[AdapterSpec], bias: torch.Tensor | None = None):
        super().__init__()
        w = self._setup(weight, bias)
        self.register_buffer("weight", w)
        self._pack_adapters(adapters, w)

    def forward(self, x: torch.Tensor, adapter_ids: Sequence[str]) -> torch.Tensor:
        from . import ops

        xp = self._prep(x, adapter_ids)
        ten = torch.tensor([self.adapter_index[a] for a in adapter_ids], dtype=torch.int32, device=x.device)
        y = ops.lora_linear(xp, self.weight[None], bias=self.bias, row_tenant=ten, n_tenants=len(self.adapter_order),
                            rank=self.rank_pad, lora_a=self.lora_a, lora_b=self.lora_b, lora_scale=self.lora_scale)
        return y[:, : self.out_features]


class StageMLAdapterBankLinear(_DenseBase):
    """Residualized multi-adapter linear: one folded weight per adapter, grouped rows."""

    def __init__(self, weight: torch.Tensor, adapters: Sequence[AdapterSpec], bias: torch.Tensor | None = None):
        super().__init__()
        w = self._setup(weight, bias)
        self.adapter_names = [a.name for a in adapters]
        self.name_to_index = {n: i for i, n in enumerate(self.adapter_names)}
        self.register_buffer("merged_weights", self._fold(w, adapters).contiguous() if adapters else w[None, :0])

    @classmethod
    def from_lora_factors(cls, weight: torch.Tensor, adapters: Sequence[AdapterSpec], bias: torch.Tensor | None = None):
        return cls(weight, adapters, bias)

    def forward(self, x: torch.Tensor, adapter_ids: Sequence[str]) -> torch.Tensor:
        from . import ops

        xp = self._prep(x, adapter_ids)
        grp = torch.tensor([self.name_to_index[a] for a in adapter_ids], dtype=torch.int32, device=x.device)
        y = ops.lora_linear(xp, self.merged_weights, bias=self.bias, row_group=grp)
        return y[:, : self.out_features]


class OnTheFlyMergeLinear(_DenseBase):
    """Slow baseline: merges the adapters present in the batch on every call."""

    def __init__(self, weight: torch.Tensor, adapters: Sequence[AdapterSpec], bias: torch.Tensor | None = None):
        super().__init__()
        w = self._setup(weight, bias)
        self.register_buffer("weight", w)
        self.adapters = {a.name: a for a in adapters}

    def forward(self, x: torch.Tensor, adapter_ids: Sequence[str]) -> torch.Tensor:
        from . import ops

        xp = self._prep(x, adapter_ids)
        present = sorted(set(adapter_ids))
        merged = self._fold(self.weight, [self.adapters[n] for n in present])
        idx = {n: i for i, n in enumerate(present)}
        grp = torch.tensor([idx[a] for a in adapter_ids], dtype=torch.int32, device=x.device)
        y = ops.lora_linear(xp, merged, bias=self.bias, row_group=grp)
        return y[:, : self.out_features]


def make_random_adapters(*, num_adapters: int, in_features: int, out_features: int, rank: int, dtype: torch.dtype,
                         device: torch.device, scaling: float | None = None) -> list[AdapterSpec]:
    """Random adapters, A ~ N(0, 1/in), B ~ N(0, 1/rank), scaling 16/rank unless given (stageml/adapter_bank.py:138-156)."""
    if scaling is None:
        scaling = 16.0 / float(rank)
    out = []
    for i in range(num_adapters):
        A = torch.randn(rank, in_features, device=device, dtype=dtype) / (in_features ** 0.5)
        B = torch.randn(out_features, rank, device=device, dtype=dtype) / (rank ** 0.5)
        out.append(AdapterSpec(name=f"adapter_{i}", A=A, B=B, scaling=float(scaling)))
    return out


def make_adapter_ids(batch: int, num_adapters: int, pattern: str = "round_robin") -> list[str]:
    """Per-row adapter names: single, round_robin or clustered (stageml/adapter_bank.py:159-170)."""
    if pattern == "single":
        return ["adapter_0"] * batch
    if pattern == "round_robin":
        return [f"adapter_{i % num_adapters}" for i in range(batch)]
    if pattern == "clustered":
        group = max(1, batch // num_adapters)
        return [f"adapter_{min(i // group, num_adapters - 1)}" for i in range(batch)]
    raise ValueError(f"unknown adapter id pattern: {pattern}")


__all__ = ["AdapterSpec", "DynamicLoRALinear", "StageMLAdapterBankLinear", "OnTheFlyMergeLinear",
           "make_random_adapters", "make_adapter_ids"]
