"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference implementation itself (uwm-se/stageML, read from the path
given by --reference, a required argument) on small seeded inputs and
stores inputs and outputs as .npz files next to this script. Only this
generator reads the reference; the tests read the committed .npz files.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference PATH

Cases (reference file the outputs come from):
  moe_lora_layers.npz    DynamicMoELoRALayer / MaterializedMoELoRALayer (stageml/moe_lora_layers.py),
                         setup of tests/test_moe_lora_correctness.py
  adapter_bank.npz       DynamicLoRALinear / StageMLAdapterBankLinear / OnTheFlyMergeLinear
                         (stageml/adapter_bank.py), setup of tests/test_adapter_bank.py
  adapter_cache.npz      choose_hot_adapters + StageMLCostBasedAdapterCache (stageml/adapter_cache.py)
  fold.npz               materialize_residual_weight (stageml/triton_generator.py), known answer + random
  fallback_moe.npz       _fallback_moe (stageml/custom_op_registry.py)
  request_executor.npz   RequestExecutor.dynamic_one / bta_one (benchmarks/multitenant_bta_system_bench.py)
  routing.npz            make_routing (benchmarks/real_moe_lora_residual_bench.py) with a small gate module
  tenants.npz            sample_tenants (benchmarks/multitenant_bta_system_bench.py)
  single_lora.npz        trace_and_annotate -> optimize_evaluation_order -> specialize on the config-1
                         LoRA expression y = x W + s (x A) B (stageml/tracer.py, rewrite.py, evaluator.py)
  router_split.npz       route_fused_experts with fake backends (stageml/vllm_stage_router.py)
  workload_plan.npz      make_workload_plan (benchmarks/multitenant_bta_system_bench.py), every
                         materialization policy
  residual_plan.json     choose_residual_plan + plan_to_json (stageml/residual_planner.py,
                         stageml/moe_plan_export.py) for a seeded set of adapters
  expert_lora_adapter.npz  load_expert_lora_adapter (benchmarks/real_moe_lora_residual_bench.py) on
                         a seeded PEFT-style checkpoint (the state dict is stored too)

    python tests/golden/make_golden.py --only workload_plan         # that case alone
    python tests/golden/make_golden.py --only expert_lora_adapter
    python tests/golden/make_golden.py --only residual_plan
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def np32(t):
    return t.detach().cpu().to(dtype=__import__("torch").float32).numpy()


PLAN_CASES = [  # (policy, distribution, seed)
    ("none", "zipf", 5), ("all", "uniform", 6), ("top_k", "zipf", 7), ("memory_budget", "bursty", 8),
    ("top_k", "round_robin", 9),
]
PLAN_ARGS = dict(num_requests=40, num_tenants=12, num_adapters=5, tokens_available=256, tokens_per_request=16,
                 zipf_alpha=1.1, burst_size=3, materialize_top_k=3, materialize_min_requests=2, memory_budget_mb=1.0,
                 memory_per_adapter_bytes=300000)


def workload_plan() -> None:
    import multitenant_bta_system_bench as mb

    out = {}
    for i, (policy, dist, seed) in enumerate(PLAN_CASES):
        plan = mb.make_workload_plan(distribution=dist, materialization_policy=policy, seed=seed, **PLAN_ARGS)
        out[f"c{i}_requests"] = np.array([[r.request_id, r.tenant_id, r.adapter_id, r.start, r.end]
                                          for r in plan.requests])
        out[f"c{i}_materialized"] = np.array(sorted(plan.materialized_adapter_ids), dtype=np.int64)
        out[f"c{i}_selected_bytes"] = np.array(plan.selected_materialized_memory_bytes)
    np.savez(HERE / "workload_plan.npz", **out)


def adapter_state_dict(seed: int = 21):
    """A PEFT-style Mixtral expert LoRA state dict: 4 experts x (w1, w3, w2) x (A, B) at
    rank 4, one expert at rank 2, one without its w1 B, plus attention LoRA keys."""
    import torch

    g = torch.Generator().manual_seed(seed)
    E, H, I = 4, 16, 24
    sd = {}
    pre = "base_model.model.model.layers.0.block_sparse_moe.experts"
    for e in range(E):
        r = 2 if e == 3 else 4
        for proj, (din, dout) in (("w1", (H, I)), ("w3", (H, I)), ("w2", (I, H))):
            sd[f"{pre}.{e}.{proj}.lora_A.default.weight"] = torch.randn(r, din, generator=g)
            if not (e == 2 and proj == "w1"):
                sd[f"{pre}.{e}.{proj}.lora_B.default.weight"] = torch.randn(dout, r, generator=g)
    sd["base_model.model.model.layers.0.self_attn.q_proj.lora_A.default.weight"] = torch.randn(4, H, generator=g)
    sd["base_model.model.model.layers.0.self_attn.q_proj.lora_B.default.weight"] = torch.randn(H, 4, generator=g)
    return sd, E, H, I


def expert_lora_adapter() -> None:
    import tempfile

    import real_moe_lora_residual_bench as rb
    from safetensors.torch import save_file

    sd, E, H, I = adapter_state_dict()
    out = {"keys": np.array(sorted(sd)), "E": np.array(E), "H": np.array(H), "I": np.array(I)}
    for i, k in enumerate(sorted(sd)):
        out[f"t{i}"] = sd[k].numpy()
    with tempfile.TemporaryDirectory() as d:
        save_file(sd, os.path.join(d, "adapter_model.safetensors"))
        for proj, (din, dout) in (("w1", (H, I)), ("w3", (H, I)), ("w2", (I, H))):
            os.environ["LORA_PROJECTION"] = proj
            spec = rb.load_expert_lora_adapter(Path(d), num_experts=E, in_features=din, out_features=dout)
            out[f"{proj}_A"] = spec.A.numpy()
            out[f"{proj}_B"] = spec.B.numpy()
            out[f"{proj}_scaling"] = np.array(spec.scaling)
        os.environ.pop("LORA_PROJECTION", None)
    np.savez(HERE / "expert_lora_adapter.npz", **out)


def residual_plan() -> None:
    from stageml.moe_ir import MoEAdapterMeta
    from stageml.moe_plan_export import plan_to_json
    from stageml.residual_planner import AdapterQuantInfo, PlannerConfig, choose_residual_plan

    metas = [MoEAdapterMeta(f"adapter_{i}", rank=r, num_experts=8, in_features=4096, out_features=14336,
                            dtype="bf16", request_count=c)
             for i, (r, c) in enumerate([(16, 900), (16, 450), (8, 120), (32, 600), (64, 700), (16, 40), (16, 300)])]
    cfg = PlannerConfig(memory_budget_mb=2000.0, dtype="bf16", hot_request_threshold=200,
                        disaggregate_request_threshold=500, rank_specialization_threshold=16)
    quant = {"adapter_6": AdapterQuantInfo(epsilon=0.5, safe=True)}
    (HERE / "residual_plan.json").write_text(plan_to_json(choose_residual_plan(metas, config=cfg,
                                                                               quant_info=quant)) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference project (read only)")
    ap.add_argument("--only", default=None, help="generate one case (workload_plan)")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "benchmarks"))
    if args.only == "workload_plan":
        workload_plan()
        return
    if args.only == "expert_lora_adapter":
        expert_lora_adapter()
        return
    if args.only == "residual_plan":
        residual_plan()
        return
    import torch
    import torch.nn as nn

    torch.set_num_threads(4)

    # ---------------------------------------------------------------- moe_lora_layers
    from stageml.moe_lora_layers import (DynamicMoELoRALayer, MaterializedMoELoRALayer, make_random_moe_adapters,
                                         make_round_robin_adapter_ids, normalize_routing_weights)

    torch.manual_seed(0)
    E, din, dout, nA, k, T = 4, 8, 6, 3, 2, 7
    W = torch.randn(E, dout, din)
    ads = make_random_moe_adapters(num_adapters=nA, num_experts=E, in_features=din, out_features=dout, ranks=[2, 3],
                                   dtype=torch.float32, device=torch.device("cpu"))
    x = torch.randn(T, din)
    ids = torch.tensor([[i % E, (i + 1) % E] for i in range(T)], dtype=torch.long)
    rw = normalize_routing_weights(ids)
    aids = make_round_robin_adapter_ids(T, nA)
    y_dyn = DynamicMoELoRALayer(W, ads)(x, ids, rw, aids)
    mat = MaterializedMoELoRALayer(W, ads)
    y_mat = mat(x, ids, rw, aids)
    out = dict(x=np32(x), W=np32(W), ids=ids.numpy(), rw=np32(rw), adapter_idx=np.array([i % nA for i in range(T)]),
               scaling=np.array([a.scaling for a in ads], dtype=np.float64), y_dyn=np32(y_dyn), y_mat=np32(y_mat),
               merged=np32(mat.merged_weight))
    for i, a in enumerate(ads):
        out[f"A{i}"] = np32(a.A)
        out[f"B{i}"] = np32(a.B)
    np.savez(HERE / "moe_lora_layers.npz", **out)

    # ---------------------------------------------------------------- adapter_bank
    from stageml.adapter_bank import (DynamicLoRALinear, OnTheFlyMergeLinear, StageMLAdapterBankLinear,
                                      make_adapter_ids, make_random_adapters)

    torch.manual_seed(0)
    Wd = torch.randn(8, 8)
    bias = torch.randn(8)
    ads = make_random_adapters(num_adapters=3, in_features=8, out_features=8, rank=2, dtype=torch.float32,
                               device=torch.device("cpu"))
    x = torch.randn(6, 8)
    names = make_adapter_ids(6, 3, "round_robin")
    out = dict(x=np32(x), W=np32(Wd), bias=np32(bias), adapter_idx=np.array([int(n.split("_")[1]) for n in names]),
               scaling=np.array([a.scaling for a in ads]),
               y_dyn=np32(DynamicLoRALinear(Wd, ads, bias)(x, names)),
               y_bank=np32(StageMLAdapterBankLinear(Wd, ads, bias)(x, names)),
               y_otf=np32(OnTheFlyMergeLinear(Wd, ads, bias)(x, names)))
    for i, a in enumerate(ads):
        out[f"A{i}"] = np32(a.A)
        out[f"B{i}"] = np32(a.B)
    np.savez(HERE / "adapter_bank.npz", **out)

    # ---------------------------------------------------------------- adapter_cache
    from stageml.adapter_cache import StageMLCostBasedAdapterCache, choose_hot_adapters
    from multitenant_bta_system_bench import sample_tenants

    torch.manual_seed(1)
    n_in, n_out, nA, r = 24, 16, 5, 4
    Wc = torch.randn(n_out, n_in)
    ads = make_random_adapters(num_adapters=nA, in_features=n_in, out_features=n_out, rank=r, dtype=torch.float32,
                               device=torch.device("cpu"), scaling=2.0)
    rows = sample_tenants(12, nA, "zipf", 1.1, 1, 7)
    names = [f"adapter_{i}" for i in rows]
    counts = {}
    for n in names:
        counts[n] = counts.get(n, 0) + 1
    per_mb = n_in * n_out * 4 / (1024 * 1024)
    cached, decisions = choose_hot_adapters(counts, ads, in_features=n_in, out_features=n_out, dtype=torch.float32,
                                            memory_budget_mb=2 * per_mb)
    x = torch.randn(12, n_in)
    layer = StageMLCostBasedAdapterCache(Wc, ads, cached_adapter_names=cached)
    out = dict(x=np32(x), W=np32(Wc), adapter_idx=np.array(rows), scaling=np.array([a.scaling for a in ads]),
               cached=np.array([int(n.split("_")[1]) for n in cached]), budget_mb=np.array(2 * per_mb),
               y=np32(layer(x, names)),
               decision_cached=np.array([int(d.cached) for d in decisions]),
               decision_names=np.array([int(d.name.split("_")[1]) for d in decisions]))
    for i, a in enumerate(ads):
        out[f"A{i}"] = np32(a.A)
        out[f"B{i}"] = np32(a.B)
    np.savez(HERE / "adapter_cache.npz", **out)

    # ---------------------------------------------------------------- fold
    from stageml.triton_generator import materialize_residual_weight

    torch.manual_seed(2)
    Wf = torch.randn(12, 20)
    Af = torch.randn(3, 20)
    Bf = torch.randn(12, 3)
    np.savez(HERE / "fold.npz", known_W=np.zeros((3, 4), np.float32), known_A=np.ones((2, 4), np.float32),
             known_B=np.ones((3, 2), np.float32), known_scale=np.array(0.5),
             known_out=np32(materialize_residual_weight(torch.zeros(3, 4), torch.ones(2, 4), torch.ones(3, 2),
                                                        scaling=0.5)),
             W=np32(Wf), A=np32(Af), B=np32(Bf), scale=np.array(0.7),
             out=np32(materialize_residual_weight(Wf, Af, Bf, scaling=0.7)))

    # ---------------------------------------------------------------- fallback_moe
    from stageml.custom_op_registry import _fallback_moe

    g = torch.Generator().manual_seed(3)
    T, H, I, E, k = 5, 16, 8, 3, 2
    hid = torch.randn(T, H, generator=g)
    gu = torch.randn(E, 2 * I, H, generator=g) * 0.3
    dn = torch.randn(E, H, I, generator=g) * 0.3
    tid = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    tw = torch.softmax(torch.randn(T, k, generator=g), -1)
    np.savez(HERE / "fallback_moe.npz", hidden=np32(hid), gate_up=np32(gu), down=np32(dn), topk_ids=tid.numpy(),
             topk_weights=np32(tw), out=np32(_fallback_moe(hid, gu, dn, tw, tid)))

    # ---------------------------------------------------------------- request executor
    import multitenant_bta_system_bench as mb
    from stageml.moe_lora_layers import MoEAdapterSpec

    g = torch.Generator().manual_seed(4)
    T, H, I, E, k, r = 9, 16, 8, 3, 2, 4
    xr = torch.randn(T, H, generator=g)
    gu = torch.randn(E, 2 * I, H, generator=g) * 0.2
    dn = torch.randn(E, H, I, generator=g) * 0.2
    tid = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    tw = torch.softmax(torch.randn(T, k, generator=g), -1)
    ads = [MoEAdapterSpec(f"a{i}", torch.randn(E, r, H, generator=g) * 0.3, torch.randn(E, I, r, generator=g) * 0.3,
                          0.5 + 0.25 * i) for i in range(2)]
    ex = mb.RequestExecutor(gu, dn, ads, {0})
    np.savez(HERE / "request_executor.npz", x=np32(xr), gate_up=np32(gu), down=np32(dn), topk_ids=tid.numpy(),
             topk_weights=np32(tw), A0=np32(ads[0].A), B0=np32(ads[0].B), A1=np32(ads[1].A), B1=np32(ads[1].B),
             scaling=np.array([a.scaling for a in ads]),
             dyn0=np32(ex.dynamic_one(xr, tid, tw, 0)), dyn1=np32(ex.dynamic_one(xr, tid, tw, 1)),
             bta0=np32(ex.bta_one(xr, tid, tw, 0)), bta1=np32(ex.bta_one(xr, tid, tw, 1)),
             residual_gate_up0=np32(ex.residual_gate_up(0)))

    # ---------------------------------------------------------------- routing
    import real_moe_lora_residual_bench as rb

    class _Block(nn.Module):
        def __init__(self, h, e):
            super().__init__()
            self.gate = nn.Linear(h, e, bias=False)

    class _Layer(nn.Module):
        def __init__(self, h, e):
            super().__init__()
            self.block_sparse_moe = _Block(h, e)

    class _Model(nn.Module):
        def __init__(self, h, e):
            super().__init__()
            self.layers = nn.ModuleList([_Layer(h, e)])

    torch.manual_seed(5)
    Hr, Er, Tr, kr = 32, 8, 40, 2
    model = _Model(Hr, Er)
    hidden = torch.randn(Tr, Hr)
    rids, rw, _ = rb.make_routing(model, hidden, Er, kr, "cpu")
    np.savez(HERE / "routing.npz", hidden=np32(hidden), gate_w=np32(model.layers[0].block_sparse_moe.gate.weight),
             k=np.array(kr), ids=rids.numpy(), weights=np32(rw))

    # ---------------------------------------------------------------- tenants
    out = {}
    for dist in ("uniform", "zipf", "round_robin", "bursty"):
        out[dist] = np.array(mb.sample_tenants(50, 16, dist, 1.1, 3, 11))
    np.savez(HERE / "tenants.npz", **out)

    # ---------------------------------------------------------------- single LoRA (config-1 form, small)
    from stageml.evaluator import specialize
    from stageml.rewrite import optimize_evaluation_order
    from stageml.tracer import trace_and_annotate

    class SingleLoRA(nn.Module):
        def __init__(self, d_in=32, d_out=24, rank=4, alpha=8.0):
            super().__init__()
            self.W = nn.Parameter(torch.randn(d_in, d_out) / d_in ** 0.5)
            self.A = nn.Parameter(torch.randn(d_in, rank) / d_in ** 0.5)
            self.B = nn.Parameter(torch.randn(rank, d_out) / rank ** 0.5)
            self.s = alpha / rank

        def forward(self, x):
            return x @ self.W + self.s * ((x @ self.A) @ self.B)

    torch.manual_seed(6)
    m = SingleLoRA().eval()
    x = torch.randn(3, 32)
    gm, ann = trace_and_annotate(m, {"x": "stage1"})
    rew, rann, stats = optimize_evaluation_order(gm, ann)
    residual = specialize(rew, rann)
    with torch.no_grad():
        np.savez(HERE / "single_lora.npz", x=np32(x), W=np32(m.W), A=np32(m.A), B=np32(m.B), scale=np.array(m.s),
                 y=np32(m(x)), y_residual=np32(residual(x)), rewrites=np.array(stats.total_rewrites))

    # ---------------------------------------------------------------- router split
    from stageml.vllm_stage_router import StageMLTenantRouter, TenantKernel, route_fused_experts

    router = StageMLTenantRouter({0: TenantKernel(tenant_id=0, adapter_id=0, backend="t", artifact="x", symbol="s"),
                                  3: TenantKernel(tenant_id=3, adapter_id=1, backend="t", artifact="x", symbol="s")})
    hidden = torch.randn(6, 3)
    tenant_ids = torch.tensor([0, 1, 3, 2, 0, 5])
    fv = lambda h, gu, dn, *a: torch.zeros((h.shape[0], dn.shape[1])) + 1 + h[:, :1]
    fs = lambda h, gu, dn, *a: torch.zeros((h.shape[0], dn.shape[1])) + 2 + h[:, :1]
    y = route_fused_experts(hidden=hidden, gate_up=torch.randn(2, 4, 3), down=torch.randn(2, 3, 2),
                            topk_weights=torch.ones(6, 1), topk_ids=torch.zeros(6, 1, dtype=torch.long),
                            tenant_ids=tenant_ids, router=router, vllm_fused_experts=fv, stageml_op=fs)
    np.savez(HERE / "router_split.npz", hidden=np32(hidden), tenant_ids=tenant_ids.numpy(),
             materialized=np.array([0, 3]), out=np32(y))
    workload_plan()
    expert_lora_adapter()
    residual_plan()
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
