"""Request-level executor: the workload plan against the reference's own plans
(golden vectors), the w1-adapter bank packing on CPU, and (-m gpu) the executor
against the reference RequestExecutor's outputs and the batched plan against the
per-request calls."""

import numpy as np
import pytest
import torch

from conftest import load_golden, rel_l2

PLAN_CASES = [("none", "zipf", 5), ("all", "uniform", 6), ("top_k", "zipf", 7), ("memory_budget", "bursty", 8),
              ("top_k", "round_robin", 9)]
PLAN_ARGS = dict(num_requests=40, num_tenants=12, num_adapters=5, tokens_available=256, tokens_per_request=16,
                 zipf_alpha=1.1, burst_size=3, materialize_top_k=3, materialize_min_requests=2, memory_budget_mb=1.0,
                 memory_per_adapter_bytes=300000)


@pytest.mark.parametrize("i", range(len(PLAN_CASES)))
def test_workload_plan_matches_reference(i):
    from stageml_b200.executor import make_workload_plan

    g = load_golden("workload_plan")
    policy, dist, seed = PLAN_CASES[i]
    plan = make_workload_plan(distribution=dist, materialization_policy=policy, seed=seed, **PLAN_ARGS)
    got = np.array([[r.request_id, r.tenant_id, r.adapter_id, r.start, r.end] for r in plan.requests])
    np.testing.assert_array_equal(got, g[f"c{i}_requests"])
    np.testing.assert_array_equal(np.array(sorted(plan.materialized_adapter_ids), dtype=np.int64),
                                  g[f"c{i}_materialized"])
    assert plan.selected_materialized_memory_bytes == int(g[f"c{i}_selected_bytes"])


def test_pack_w1_adapters_layout():
    from stageml_b200.executor import pack_w1_adapters
    from stageml_b200.moe_lora_layers import MoEAdapterSpec

    E, I, H = 3, 24, 32
    ads = [MoEAdapterSpec(f"a{i}", torch.randn(E, r, H), torch.randn(E, I, r), 0.5 + i) for i, r in enumerate((4, 8))]
    a13, b13, sc, rp = pack_w1_adapters(ads, I, H, torch.float32, "cpu")
    assert rp == 8 and a13.shape == (2, E, 16, H) and b13.shape == (2, E, 2 * I, 8)
    assert torch.equal(a13[0, :, :4], ads[0].A) and not a13[0, :, 4:].any()  # w1 rows, then zeros (w3 rows too)
    assert torch.equal(b13[1, :, :I], ads[1].B) and not b13[:, :, I:].any()
    assert sc.tolist() == [0.5, 1.5]
    # w1 LoRA through the bank equals the adapter's own product
    x = torch.randn(5, H)
    s = x @ a13[0, 1, :8].t()
    assert torch.allclose(s @ b13[0, 1, :I].t(), x @ ads[0].A[1].t() @ ads[0].B[1].t(), atol=1e-4)


# ------------------------------------------------------------------ GPU
def _golden_executor(dtype=torch.bfloat16):
    from stageml_b200.executor import RequestExecutor
    from stageml_b200.moe_lora_layers import MoEAdapterSpec

    g = load_golden("request_executor")
    d = lambda n: torch.from_numpy(g[n]).to("cuda", dtype)
    ads = [MoEAdapterSpec(f"a{i}", d(f"A{i}"), d(f"B{i}"), float(g["scaling"][i])) for i in range(2)]
    ex = RequestExecutor(d("gate_up"), d("down"), ads, {0})
    return g, ex, d("x"), torch.from_numpy(g["topk_ids"]).cuda(), torch.from_numpy(g["topk_weights"]).cuda()


@pytest.mark.gpu
def test_executor_matches_reference_request_executor():
    g, ex, x, ids, w = _golden_executor()
    f = lambda t: t.float().cpu().numpy().astype(np.float64)
    for a in (0, 1):
        # includes the bf16 rounding of the reference's fp32 inputs
        assert rel_l2(f(ex.dynamic_one(x, ids, w, a)), g[f"dyn{a}"]) < 3e-2
        assert rel_l2(f(ex.bta_one(x, ids, w, a)), g[f"bta{a}"]) < 3e-2
    assert rel_l2(f(ex.residual_gate_up(0)), g["residual_gate_up0"]) < 1e-2
    assert ex.compile_time_ms >= 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("policy", ["none", "top_k"])
def test_batched_plan_matches_per_request(policy):
    from stageml_b200.executor import RequestExecutor, make_workload_plan, run_sequence
    from stageml_b200.moe_lora_layers import MoEAdapterSpec

    torch.manual_seed(0)
    dev, dt = "cuda", torch.bfloat16
    T, H, I, E, k, nA, r = 512, 256, 384, 6, 2, 5, 16
    hidden = torch.randn(T, H, device=dev).to(dt)
    gate_up = (torch.randn(E, 2 * I, H, device=dev) * H ** -0.5).to(dt)
    down = (torch.randn(E, H, I, device=dev) * I ** -0.5).to(dt)
    ids = torch.stack([torch.randperm(E, device=dev)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, device=dev), -1)
    ads = [MoEAdapterSpec(f"a{i}", (torch.randn(E, r, H, device=dev) * H ** -0.5).to(dt),
                          (torch.randn(E, I, r, device=dev) * r ** -0.5).to(dt), 0.5 + 0.25 * i) for i in range(nA)]
    plan = make_workload_plan(num_requests=30, num_tenants=9, num_adapters=nA, tokens_available=T,
                              tokens_per_request=24, distribution="zipf", zipf_alpha=1.1, burst_size=1,
                              materialization_policy=policy, materialize_top_k=2, materialize_min_requests=1,
                              memory_budget_mb=0, memory_per_adapter_bytes=0, seed=3)
    ex = RequestExecutor(gate_up, down, ads, plan.materialized_adapter_ids)
    y, off = ex.run_batched(plan, hidden, ids, w)
    for q, req in enumerate(plan.requests):
        x = hidden[req.start:req.end]
        ref = ex.dynamic_one(x, ids[req.start:req.end], w[req.start:req.end], req.adapter_id).float()
        assert rel_l2(y[off[q]:off[q + 1]].float().cpu().numpy(), ref.cpu().numpy()) < 1e-2, q
        bta = ex.bta_one(x, ids[req.start:req.end], w[req.start:req.end], req.adapter_id).float()
        assert rel_l2(bta.cpu().numpy(), ref.cpu().numpy()) < 2e-2, q
    c_b = run_sequence(ex, plan, hidden, ids, w, "batched")
    c_d = run_sequence(ex, plan, hidden, ids, w, "dynamic")
    assert abs(float(c_b) - float(c_d)) <= 1e-2 * max(1.0, abs(float(c_d)))
