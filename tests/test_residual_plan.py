"""Residual plans: the reference planner's JSON (tests/golden/residual_plan.json,
written by choose_residual_plan + plan_to_json) read back, and (-m gpu) the
planned layer against the all-dynamic layer."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import rel_l2

GOLDEN = Path(__file__).resolve().parent / "golden" / "residual_plan.json"


def test_read_reference_plan_json():
    from stageml_b200.residual_plan import read_residual_plan

    data = json.loads(GOLDEN.read_text())
    for src in (GOLDEN, GOLDEN.read_text(), data):
        plan = read_residual_plan(src)
        assert plan.by_kind() == data["summary"]
        assert plan.used_memory_bytes == data["used_memory_bytes"] and plan.theta == data["theta"]
        assert [(p.adapter, p.kind, p.rank) for p in plan.plans] == [(p["adapter"], p["kind"], p["rank"])
                                                                      for p in data["plans"]]
        assert plan.materialized() == {"adapter_0": {"all"}, "adapter_4": {"all"}}
    bad = dict(data, plans=[dict(data["plans"][0], kind="jit")])
    with pytest.raises(ValueError):
        read_residual_plan(bad)


@pytest.mark.gpu
def test_planned_layer_matches_dynamic():
    from stageml_b200 import ops
    from stageml_b200.executor import pack_w1_adapters
    from stageml_b200.moe_lora_layers import MoEAdapterSpec
    from stageml_b200.residual_plan import PlannedMoELayer, read_residual_plan

    torch.manual_seed(0)
    dev, dt = "cuda", torch.bfloat16
    T, H, I, E, k, nA, r = 700, 256, 384, 6, 2, 4, 16
    x = torch.randn(T, H, device=dev).to(dt)
    gate_up = (torch.randn(E, 2 * I, H, device=dev) * H ** -0.5).to(dt)
    down = (torch.randn(E, H, I, device=dev) * I ** -0.5).to(dt)
    ids = torch.stack([torch.randperm(E, device=dev)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, device=dev), -1)
    ads = [MoEAdapterSpec(f"adapter_{i}", (torch.randn(E, r, H, device=dev) * H ** -0.5).to(dt),
                          (torch.randn(E, I, r, device=dev) * r ** -0.5).to(dt), 1.0 + 0.5 * i) for i in range(nA)]
    entry = lambda a, e, kind: {"adapter": a, "expert": e, "kind": kind, "rank": r, "memory_bytes": 0,
                                "estimated_latency_cost": 0.0, "epsilon": 0.0, "reason": ""}
    plan = read_residual_plan({"plans": [entry("adapter_1", "all", "materialized_residual"),
                                         entry("adapter_2", 1, "materialized_residual"),
                                         entry("adapter_2", 4, "materialized_residual"),
                                         entry("adapter_0", "all", "non_materializing_fusion"),
                                         entry("adapter_3", "all", "fallback")]})
    layer = PlannedMoELayer(gate_up, down, ads, plan)
    ten = torch.randint(-1, nA, (T,), device=dev, dtype=torch.int32)
    y = layer(x, ids, w, ten)
    a13, b13, sc, rp = pack_w1_adapters(ads, I, H, dt, dev)
    ref = ops.moe_forward(x, gate_up, down, topk_ids=ids, topk_weights=w, tenant_ids=ten, n_tenants=nA, rank=rp,
                          lora_a13=a13, lora_b13=b13, lora_scale=sc)
    assert rel_l2(y.float().cpu().numpy(), ref.float().cpu().numpy()) < 2e-2
    assert ops.take_status(x) == 0
    man = layer.kernel_manifest()
    assert [(e.tenant_id, e.artifact) for e in man.entries] == [(1, "folded:adapter_1:experts=0,1,2,3,4,5"),
                                                                 (2, "folded:adapter_2:experts=1,4")]
    assert layer.compile_time_ms >= 0.0
