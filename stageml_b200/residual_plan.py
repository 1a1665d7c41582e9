"""Residual plans -> folded weights on the device and the layer that serves them.

``read_residual_plan`` reads the JSON the reference's planner writes
(``choose_residual_plan`` + ``plan_to_json``; stageml/residual_planner.py:48-153,
stageml/moe_plan_export.py:9-17, format of ``ResidualPlan.to_dict`` in
stageml/moe_ir.py): one entry per (adapter, expert | "all") with its kind.

``PlannedMoELayer`` executes such a plan for a SwiGLU MoE layer whose adapters
apply LoRA to w1 (as the reference's request executor):

* ``materialized_residual`` entries are folded at construction (stage 0, on the
  device): the adapter's w1 delta s * B @ A is added to a copy of ``gate_up`` for
  the planned experts ("all" or one expert per entry);
* every other kind (``non_materializing_fusion``, ``dynamic``, ``fallback``, and
  ``disaggregated``, which the reference's artifact does not execute) runs the
  adapter dynamically on the fused LoRA path of the grouped GEMMs.

A call takes per-token adapter ids. Tokens of an adapter with folded experts run
on its folded ``gate_up``, with the LoRA of its other experts still applied
dynamically (their bank slices stay, the folded experts' are zero); all other
tokens run as one dynamic call. Outputs come back in token order.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

from . import ops
from .executor import pack_w1_adapters
from .moe_lora_layers import MoEAdapterSpec
from .vllm_stage_router import KernelManifest, KernelManifestEntry

__all__ = ["PlanEntry", "ResidualPlanSpec", "read_residual_plan", "PlannedMoELayer", "MATERIALIZED"]

MATERIALIZED = "materialized_residual"
KINDS = ("dynamic", "non_materializing_fusion", MATERIALIZED, "disaggregated", "fallback")


@dataclass(frozen=True)
class PlanEntry:
    adapter: str
    expert: int | str
    kind: str
    rank: int
    memory_bytes: int
    estimated_latency_cost: float
    epsilon: float
    reason: str


@dataclass(frozen=True)
class ResidualPlanSpec:
    plans: tuple[PlanEntry, ...]
    memory_budget_bytes: int
    used_memory_bytes: int
    theta: float
    metadata: dict[str, Any] = field(default_factory=dict)

    def by_kind(self) -> dict[str, int]:
        out: dict[str, int] = {}
        for p in self.plans:
            out[p.kind] = out.get(p.kind, 0) + 1
        return out

    def materialized(self) -> dict[str, set]:
        """adapter -> {"all"} or the set of expert ids to fold."""
        out: dict[str, set] = {}
        for p in self.plans:
            if p.kind == MATERIALIZED:
                out.setdefault(p.adapter, set()).add(p.expert)
        return out


def read_residual_plan(source) -> ResidualPlanSpec:
    """A plan from a JSON file path, a JSON string or the parsed dict."""
    if isinstance(source, dict):
        data = source
    else:
        text = str(source)
        data = json.loads(text if text.lstrip().startswith("{") else Path(text).read_text())
    entries = []
    for p in data.get("plans", []):
        kind = str(p["kind"])
        if kind not in KINDS:
            raise ValueError(f"unknown plan kind {kind!r}")
        expert = p.get("expert", "all")
        entries.append(PlanEntry(adapter=str(p["adapter"]), expert=expert if expert == "all" else int(expert),
                                 kind=kind, rank=int(p.get("rank", 0)), memory_bytes=int(p.get("memory_bytes", 0)),
                                 estimated_latency_cost=float(p.get("estimated_latency_cost", 0.0)),
                                 epsilon=float(p.get("epsilon", 0.0)), reason=str(p.get("reason", ""))))
    return ResidualPlanSpec(plans=tuple(entries), memory_budget_bytes=int(data.get("memory_budget_bytes", 0)),
                            used_memory_bytes=int(data.get("used_memory_bytes", 0)),
                            theta=float(data.get("theta", 0.0)), metadata=dict(data.get("metadata", {})))


class PlannedMoELayer:
    """``gate_up [E, 2I, H]``, ``down [E, H, I]`` (CUDA, 16-bit) serving the w1 adapters
    ``adapters`` (adapter id i = ``adapters[i]``, matched to plan entries by name)."""

    def __init__(self, gate_up: torch.Tensor, down: torch.Tensor, adapters: list[MoEAdapterSpec],
                 plan: ResidualPlanSpec) -> None:
        if not gate_up.is_cuda:
            raise RuntimeError("PlannedMoELayer runs on CUDA tensors (no CPU path)")
        self.gate_up = gate_up.contiguous()
        self.down = down.contiguous()
        self.adapters = adapters
        self.plan = plan
        E = int(gate_up.shape[0])
        self.intermediate = I = int(gate_up.shape[1] // 2)
        names = {a.name: i for i, a in enumerate(adapters)}
        mat = plan.materialized()
        unknown = sorted(set(mat) - set(names))
        if unknown:
            raise ValueError(f"plan names adapters that were not given: {unknown}")
        self.lora_a13, self.lora_b13, self.lora_scale, self.rank = pack_w1_adapters(
            adapters, I, int(gate_up.shape[2]), gate_up.dtype, gate_up.device)
        self.folded: dict[int, torch.Tensor] = {}  # adapter id -> gate_up with its planned experts folded
        self.folded_experts: dict[int, list[int]] = {}
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for name, experts in mat.items():
            a = names[name]
            ex = list(range(E)) if "all" in experts else sorted(int(e) for e in experts)
            if any(not 0 <= e < E for e in ex):
                raise ValueError(f"plan folds expert ids outside [0, {E}) for {name}")
            ad = adapters[a]
            dev, dt = gate_up.device, gate_up.dtype
            g = self.gate_up.clone()
            idx = torch.tensor(ex, device=dev)
            w1 = ops.lora_fold(self.gate_up[idx, :I], ad.A[idx].to(dev, dt), ad.B[idx].to(dev, dt),
                               float(ad.scaling))
            g[idx, :I] = w1
            self.folded[a] = g
            self.folded_experts[a] = ex
            self.lora_a13[a, idx] = 0  # the folded experts take no dynamic LoRA for this adapter
        e1.record()
        torch.cuda.synchronize()
        self.compile_time_ms = e0.elapsed_time(e1)
        n = len(adapters)
        slot = torch.full((n + 1,), -1, dtype=torch.int64)
        for j, a in enumerate(sorted(self.folded)):
            slot[a] = j
        self._order = sorted(self.folded)
        self._slot = slot.to(gate_up.device)  # adapter id -> folded slot (index n: tokens without an adapter)

    def _call(self, gate_up, x, ids, w, ten):
        return ops.moe_forward(x, gate_up, self.down, topk_ids=ids, topk_weights=w, tenant_ids=ten,
                               n_tenants=len(self.adapters), rank=self.rank, lora_a13=self.lora_a13,
                               lora_b13=self.lora_b13, lora_scale=self.lora_scale)

    def __call__(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                 adapter_ids: torch.Tensor) -> torch.Tensor:
        """Layer output for tokens x with their routing and adapter ids (-1: base weights only).

        The host reads one small vector (tokens per folded adapter) to size the sub-batches."""
        ten = adapter_ids.to(torch.int32)
        if not self.folded:
            return self._call(self.gate_up, x, topk_ids, topk_weights, ten)
        n = len(self.adapters)
        known = (ten >= 0) & (ten < n)  # other ids: the dynamic call reports them in the status word
        slots = self._slot[torch.where(known, ten.long(), torch.full_like(ten.long(), n))]
        nslot = len(self._order)
        counts = torch.bincount(slots + 1, minlength=nslot + 1).cpu().tolist()  # [dynamic, folded slots...]
        order = torch.argsort(slots, stable=True)  # dynamic tokens first, then each folded adapter's
        out = torch.empty((x.shape[0], self.down.shape[1]), dtype=x.dtype, device=x.device)
        start = 0
        for j, c in enumerate(counts):
            if c == 0:
                continue
            idx = order[start:start + c]
            start += c
            gu = self.gate_up if j == 0 else self.folded[self._order[j - 1]]
            out[idx] = self._call(gu, x.index_select(0, idx), topk_ids.index_select(0, idx),
                                  topk_weights.index_select(0, idx), ten.index_select(0, idx))
        return out

    def kernel_manifest(self, model: str = "moe") -> KernelManifest:
        """Tenant (= adapter id) -> folded-weights entry for the tenant router, one per folded adapter."""
        entries = tuple(KernelManifestEntry(tenant_id=a, adapter_id=a, backend="stageml_b200",
                                            artifact=f"folded:{self.adapters[a].name}:experts="
                                                     + ",".join(map(str, self.folded_experts[a])))
                        for a in self._order)
        return KernelManifest(version=1, model=model, entries=entries)
