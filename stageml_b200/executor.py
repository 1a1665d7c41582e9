"""Request-level executor of the multi-tenant MoE-LoRA layer.

Same surface as the request executor of the reference's system benchmark
(``RequestSpec``, ``WorkloadPlan``, ``make_workload_plan``, ``RequestExecutor``,
``run_sequence``; benchmarks/multitenant_bta_system_bench.py:53-72, 112-166,
379-466): a stream of requests, each a token range of one tenant, whose adapter
applies LoRA to w1 (the SiLU branch, rows ``[:I]`` of ``gate_up``) of every
expert. The per-request modes keep the reference's one-call-per-request shape:

* ``dynamic``: the request's adapter on the fly (``RequestExecutor.dynamic_one``);
* ``bta``: materialized adapters use their stage-0 folded residual weights,
  the others run dynamically (``RequestExecutor.bta_one``);
* ``vllm``: a caller-supplied fused-experts function (vLLM's keyword
  convention) on the folded weights.

``batched`` runs the whole plan as ONE layer call: the requests' token rows are
gathered once, every row carries its request's adapter id as its tenant, and
the kernels sort rows by (expert, adapter) and apply each adapter to its rows
(dynamic LoRA for every adapter -- folding cannot be batched across adapters
that share the experts' base weights). CUDA tensors only; no CPU fallback.
"""

from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from typing import Any, Callable

import torch

from . import ops
from ._packing import padded_rank
from .moe_lora_layers import MoEAdapterSpec
from .workloads import sample_tenants

__all__ = ["RequestSpec", "WorkloadPlan", "make_workload_plan", "RequestExecutor", "run_sequence",
           "pack_w1_adapters"]


@dataclass(frozen=True)
class RequestSpec:
    request_id: int
    tenant_id: int
    adapter_id: int
    start: int
    end: int


@dataclass(frozen=True)
class WorkloadPlan:
    requests: list[RequestSpec]
    tenant_request_counts: dict[int, int]
    tenant_to_adapter: dict[int, int]
    materialized_adapter_ids: set[int]
    materialization_policy: str
    estimated_memory_per_adapter_bytes: int
    selected_materialized_memory_bytes: int


def make_workload_plan(*, num_requests: int, num_tenants: int, num_adapters: int, tokens_available: int,
                       tokens_per_request: int, distribution: str, zipf_alpha: float, burst_size: int,
                       materialization_policy: str, materialize_top_k: int, materialize_min_requests: int,
                       memory_budget_mb: float, memory_per_adapter_bytes: int, seed: int) -> WorkloadPlan:
    """Requests with tenants drawn by ``sample_tenants``, tenant t served by adapter
    t % num_adapters, request r covering tokens [(r * tpr) % span, ... + tpr), and the
    adapters to materialize under the policy ("none", "all", "top_k": the most requested
    adapters with at least materialize_min_requests requests, up to materialize_top_k;
    "memory_budget": those candidates while their folded weights fit the budget)."""
    tenants = sample_tenants(num_requests, num_tenants, distribution, zipf_alpha, burst_size, seed)
    tenant_to_adapter = {t: t % num_adapters for t in range(num_tenants)}
    counts = Counter(tenants)
    adapter_counts = Counter(tenant_to_adapter[t] for t in tenants)
    if materialization_policy == "none":
        selected: list[int] = []
    elif materialization_policy == "all":
        selected = sorted(adapter_counts)
    elif materialization_policy in ("top_k", "memory_budget"):
        cand = [a for a, c in adapter_counts.most_common() if c >= materialize_min_requests]
        if materialize_top_k >= 0:
            cand = cand[:materialize_top_k]
        if materialization_policy == "top_k":
            selected = cand
        else:
            selected, used, budget = [], 0, int(memory_budget_mb * 1024 * 1024)
            for a in cand:
                if used + memory_per_adapter_bytes <= budget:
                    selected.append(a)
                    used += memory_per_adapter_bytes
    else:
        raise ValueError(f"unknown materialization policy {materialization_policy}")
    if tokens_available < tokens_per_request:
        raise ValueError("tokens_available must be at least tokens_per_request")
    span = max(1, tokens_available - tokens_per_request + 1)
    requests = []
    for rid, t in enumerate(tenants):
        start = (rid * tokens_per_request) % span
        requests.append(RequestSpec(rid, t, tenant_to_adapter[t], start, start + tokens_per_request))
    return WorkloadPlan(requests=requests, tenant_request_counts=dict(counts), tenant_to_adapter=tenant_to_adapter,
                        materialized_adapter_ids=set(selected), materialization_policy=materialization_policy,
                        estimated_memory_per_adapter_bytes=memory_per_adapter_bytes,
                        selected_materialized_memory_bytes=len(selected) * memory_per_adapter_bytes)


def pack_w1_adapters(adapters: list[MoEAdapterSpec], intermediate: int, hidden: int, dtype, device):
    """Adapter banks of the MoE layer for LoRA on w1 only: ``lora_a13 [n, E, 2r, H]``
    (rows [0, rank) = A, the w3 rows zero), ``lora_b13 [n, E, 2I, r]`` (rows [0, I) = B,
    the w3 rows zero), ``scale [n]``, with r the common rank padded to 8, 16 or 32."""
    if not adapters:
        raise ValueError("at least one adapter is needed")
    E = adapters[0].num_experts
    r = max(a.rank for a in adapters)
    rp = padded_rank(r)
    n = len(adapters)
    a13 = torch.zeros((n, E, 2 * rp, hidden), dtype=dtype, device=device)
    b13 = torch.zeros((n, E, 2 * intermediate, rp), dtype=dtype, device=device)
    for i, ad in enumerate(adapters):
        if ad.num_experts != E or tuple(ad.A.shape[2:]) != (hidden,) or tuple(ad.B.shape[1:2]) != (intermediate,):
            raise ValueError(f"adapter {ad.name}: A [E, r, {hidden}] and B [E, {intermediate}, r] expected")
        a13[i, :, : ad.rank] = ad.A.to(device=device, dtype=dtype)
        b13[i, :, :intermediate, : ad.rank] = ad.B.to(device=device, dtype=dtype)
    scale = torch.tensor([float(a.scaling) for a in adapters], dtype=torch.float32, device=device)
    return a13, b13, scale, rp


class RequestExecutor:
    """One MoE layer (``gate_up [E, 2I, H]``, ``down [E, H, I]``) serving w1 adapters.

    Materialized adapters get their folded residual ``gate_up`` (w1 + s * B @ A per
    expert) at construction (stage 0), timed in ``compile_time_ms``. The folded sets
    live after the base experts in one bank (stageml_b200/folded_sets.py): ``bta_one``
    runs a materialized adapter's requests on its sets, and the batched mode runs the
    whole stream in one call, materialized adapters' rows on their sets and every
    other row on the base experts with its adapter's LoRA.
    """

    def __init__(self, gate_up: torch.Tensor, down: torch.Tensor, adapters: list[MoEAdapterSpec],
                 materialized_ids: set[int]) -> None:
        if not gate_up.is_cuda:
            raise RuntimeError("RequestExecutor runs on CUDA tensors (no CPU path)")
        from .folded_sets import fold_w1_sets

        self.adapters = adapters
        self.materialized_ids = set(materialized_ids)
        self.intermediate = int(gate_up.shape[1] // 2)
        H = int(gate_up.shape[2])
        E = int(gate_up.shape[0])
        self.lora_a13, self.lora_b13, self.lora_scale, self.rank = pack_w1_adapters(
            adapters, self.intermediate, H, gate_up.dtype, gate_up.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        self.sets = fold_w1_sets(gate_up.contiguous(), down, adapters,
                                 [(a, list(range(E))) for a in sorted(self.materialized_ids)])
        self.residual: dict[int, torch.Tensor] = {a: self.sets.adapter_gate_up(a) for a in sorted(self.materialized_ids)}
        self._plan_rows: dict[int, tuple] = {}  # id(plan) -> (plan, rows, tenants, request of row, lengths)
        e1.record()
        torch.cuda.synchronize()
        self.compile_time_ms = e0.elapsed_time(e1)
        self.gate_up = self.sets.base_gate_up()
        self.down = self.sets.down

    def _fold(self, adapter_id: int) -> torch.Tensor:
        ad = self.adapters[adapter_id]
        I = self.intermediate
        dev, dt = self.gate_up.device, self.gate_up.dtype
        w1 = ops.lora_fold(self.gate_up[:, :I], ad.A.to(dev, dt), ad.B.to(dev, dt), float(ad.scaling))
        return torch.cat([w1, self.gate_up[:, I:]], dim=1).contiguous()

    def residual_gate_up(self, adapter_id: int) -> torch.Tensor:
        """``gate_up`` with the adapter folded into w1 (cached for materialized adapters)."""
        return self.residual[adapter_id] if adapter_id in self.residual else self._fold(adapter_id)

    def _layer(self, x, ids, weights, tenant_ids, folded: bool = False):
        """One layer call; with ``folded`` the materialized adapters' rows run on their folded sets."""
        kw = self.sets.moe_kwargs() if folded else {}
        return ops.moe_forward(x.contiguous(), self.sets.gate_up if kw else self.gate_up, self.down,
                               topk_ids=ids.contiguous(), topk_weights=weights.contiguous(), tenant_ids=tenant_ids,
                               n_tenants=len(self.adapters), rank=self.rank, lora_a13=self.lora_a13,
                               lora_b13=self.lora_b13, lora_scale=self.lora_scale, **kw)

    def dynamic_one(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, adapter_id: int) -> torch.Tensor:
        ten = torch.full((x.shape[0],), int(adapter_id), dtype=torch.int32, device=x.device)
        return self._layer(x, ids, weights, ten)

    def bta_one(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, adapter_id: int) -> torch.Tensor:
        if adapter_id not in self.residual:
            return self.dynamic_one(x, ids, weights, adapter_id)
        return ops.moe_forward(x.contiguous(), self.residual[adapter_id], self.down, topk_ids=ids.contiguous(),
                               topk_weights=weights.contiguous())

    def _rows_of(self, plan: WorkloadPlan, device):
        """Token row, adapter and request of every row of the batched call (built once per plan)."""
        hit = self._plan_rows.get(id(plan))
        if hit is not None and hit[0] is plan:
            return hit[1:]
        reqs = plan.requests
        lengths = torch.tensor([r.end - r.start for r in reqs], dtype=torch.int64)
        starts = torch.tensor([r.start for r in reqs], dtype=torch.int64)
        first = torch.repeat_interleave(torch.cumsum(lengths, 0) - lengths, lengths)
        rows = (torch.repeat_interleave(starts, lengths) + torch.arange(int(lengths.sum())) - first).to(device)
        ten = torch.repeat_interleave(torch.tensor([r.adapter_id for r in reqs], dtype=torch.int32), lengths)
        req = torch.repeat_interleave(torch.arange(len(reqs)), lengths).to(device)
        entry = (plan, rows, ten.to(device), req, lengths.to(device))
        self._plan_rows[id(plan)] = entry
        return entry[1:]

    def run_batched(self, plan: WorkloadPlan, hidden: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor):
        """All requests of the plan in one layer call; returns (outputs of the requests'
        rows in request order [sum of lengths, H], row offset of each request)."""
        if not plan.requests:
            return hidden.new_empty((0, self.down.shape[1])), [0]
        rows, ten, _, lengths = self._rows_of(plan, hidden.device)
        y = self._layer(hidden.index_select(0, rows), ids.index_select(0, rows), weights.index_select(0, rows), ten,
                        folded=True)
        offsets = [0]
        for r in plan.requests:  # from the plan on the host: no device read
            offsets.append(offsets[-1] + r.end - r.start)
        return y, offsets

    def batched_checksum(self, plan: WorkloadPlan, hidden: torch.Tensor, ids: torch.Tensor,
                         weights: torch.Tensor) -> torch.Tensor:
        """run_sequence's checksum (sum over requests of their output means) from one layer
        call, the per-request means taken by one segment reduction on the device."""
        if not plan.requests:
            return torch.zeros((), device=hidden.device, dtype=torch.float32)
        rows, ten, req, lengths = self._rows_of(plan, hidden.device)
        y = self._layer(hidden.index_select(0, rows), ids.index_select(0, rows), weights.index_select(0, rows), ten,
                        folded=True)
        sums = torch.zeros(len(plan.requests), device=y.device, dtype=torch.float32)
        sums.index_add_(0, req, y.float().sum(1))
        return (sums / (lengths.float() * y.shape[1])).sum()


def run_sequence(executor: RequestExecutor, plan: WorkloadPlan, hidden: torch.Tensor, ids: torch.Tensor,
                 weights: torch.Tensor, mode: str, *, vllm_fn: Callable[..., Any] | None = None) -> torch.Tensor:
    """Sum over the plan's requests of the mean of each request's layer output (fp32)."""
    checksum = torch.zeros((), device=hidden.device, dtype=torch.float32)
    if mode == "batched":
        return executor.batched_checksum(plan, hidden, ids, weights)
    packed: dict[int, torch.Tensor] = {}
    for req in plan.requests:
        x = hidden[req.start:req.end]
        eids = ids[req.start:req.end]
        wgts = weights[req.start:req.end]
        if mode == "dynamic":
            y = executor.dynamic_one(x, eids, wgts, req.adapter_id)
        elif mode == "bta":
            y = executor.bta_one(x, eids, wgts, req.adapter_id)
        elif mode == "vllm":
            if vllm_fn is None:
                raise RuntimeError("vLLM function was not provided")
            if req.adapter_id not in packed:
                packed[req.adapter_id] = executor.residual_gate_up(req.adapter_id)
            w1 = packed[req.adapter_id]
            y = vllm_fn(hidden_states=x.contiguous(), w1=w1, w2=executor.down, topk_weights=wgts.contiguous(),
                        topk_ids=eids.long().contiguous(), inplace=False, global_num_experts=int(w1.shape[0]))
        else:
            raise ValueError(mode)
        checksum = checksum + y.float().mean()
    return checksum
