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

A call takes per-token adapter ids and is one ``moe_forward`` launch sequence:
the folded (adapter, expert) weight sets sit after the base experts in one
``gate_up`` bank and the permutation sends each (token, expert) pair of a
folded adapter to its set (no LoRA) and every other pair to the base expert
with its adapter's LoRA (stageml_b200/folded_sets.py). Nothing is read back to
the host and the batch is never split.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

from . import ops
from .executor import pack_w1_adapters
from .folded_sets import fold_w1_sets
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
        self.folded_experts: dict[int, list[int]] = {}
        for name, experts in mat.items():
            ex = list(range(E)) if "all" in experts else sorted(int(e) for e in experts)
            if any(not 0 <= e < E for e in ex):
                raise ValueError(f"plan folds expert ids outside [0, {E}) for {name}")
            self.folded_experts[names[name]] = ex
        self._order = sorted(self.folded_experts)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        self.sets = fold_w1_sets(gate_up.contiguous(), down, adapters,
                                 [(a, self.folded_experts[a]) for a in self._order])
        e1.record()
        torch.cuda.synchronize()
        self.compile_time_ms = e0.elapsed_time(e1)
        self.gate_up = self.sets.base_gate_up()
        self.down = self.sets.down

    def __call__(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                 adapter_ids: torch.Tensor) -> torch.Tensor:
        """Layer output for tokens x with their routing and adapter ids (-1: base weights only).

        One layer call for the whole batch; ids outside [-1, len(adapters)) are reported in the
        device status word and their rows skipped."""
        return ops.moe_forward(x, self.sets.gate_up, self.down, topk_ids=topk_ids, topk_weights=topk_weights,
                               tenant_ids=adapter_ids.to(torch.int32).contiguous(), n_tenants=len(self.adapters),
                               rank=self.rank, lora_a13=self.lora_a13, lora_b13=self.lora_b13,
                               lora_scale=self.lora_scale, **self.sets.moe_kwargs())

    def kernel_manifest(self, model: str = "moe") -> KernelManifest:
        """Tenant (= adapter id) -> folded-weights entry for the tenant router, one per folded adapter."""
        entries = tuple(KernelManifestEntry(tenant_id=a, adapter_id=a, backend="stageml_b200",
                                            artifact=f"folded:{self.adapters[a].name}:experts="
                                                     + ",".join(map(str, self.folded_experts[a])))
                        for a in self._order)
        return KernelManifest(version=1, model=model, entries=entries)
