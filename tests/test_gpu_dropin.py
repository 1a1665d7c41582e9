"""The drop-in classes of stageml_b200 (same names and signatures as the reference)
on CUDA, against the reference's own outputs (golden vectors) and the oracle."""

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import lora as olora
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF = torch.bfloat16


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def bf16_round(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(BF).float().numpy().astype(np.float64)


def test_moe_lora_layers_match_reference(golden):
    from stageml_b200.moe_lora_layers import DynamicMoELoRALayer, MaterializedMoELoRALayer, MoEAdapterSpec

    g = golden("moe_lora_layers")
    n = len(g["scaling"])
    ads = [MoEAdapterSpec(f"adapter_{i}", torch.from_numpy(g[f"A{i}"]).to(DEV, BF),
                          torch.from_numpy(g[f"B{i}"]).to(DEV, BF), float(g["scaling"][i])) for i in range(n)]
    W = torch.from_numpy(g["W"]).to(DEV, BF)
    x = torch.from_numpy(g["x"]).to(DEV, BF)
    ids = torch.from_numpy(g["ids"]).to(DEV)
    rw = torch.from_numpy(g["rw"]).to(DEV)
    names = [f"adapter_{i}" for i in g["adapter_idx"]]
    y_dyn = DynamicMoELoRALayer(W, ads)(x, ids, rw, names)
    y_mat = MaterializedMoELoRALayer(W, ads)(x, ids, rw, names)
    assert y_dyn.shape == tuple(g["y_dyn"].shape)
    # oracle on the same bf16 inputs, and the reference's fp32 outputs (includes input rounding)
    r_max = max(a.rank for a in ads)
    E = W.shape[0]
    a_bank = np.zeros((n, E, r_max, W.shape[2]))
    b_bank = np.zeros((n, E, W.shape[1], r_max))
    for i, a in enumerate(ads):
        a_bank[i, :, : a.rank] = f64(a.A)
        b_bank[i, :, :, : a.rank] = f64(a.B)
    ref = omoe.moe_linear(f64(x), f64(W), g["ids"], g["rw"], tenant_ids=g["adapter_idx"], lora_a=a_bank,
                          lora_b=b_bank, lora_scale=g["scaling"])
    assert rel_l2(f64(y_dyn), ref) < 1e-2
    assert rel_l2(f64(y_mat), ref) < 1e-2
    assert rel_l2(f64(y_dyn), g["y_dyn"]) < 3e-2
    assert rel_l2(f64(y_mat), g["y_mat"]) < 3e-2


def test_moe_lora_layer_validation_errors():
    from stageml_b200.moe_lora_layers import DynamicMoELoRALayer, MoEAdapterSpec

    with pytest.raises(ValueError):
        MoEAdapterSpec("a", torch.zeros(2, 3), torch.zeros(2, 4, 3), 1.0)
    layer = DynamicMoELoRALayer(torch.zeros(2, 8, 8, device=DEV, dtype=BF), [])
    with pytest.raises(ValueError, match="token dimension"):
        layer(torch.zeros(3, 8, device=DEV, dtype=BF), torch.zeros(3, 1, dtype=torch.long, device=DEV),
              torch.ones(3, 1, device=DEV), ["a"])
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        DynamicMoELoRALayer(torch.zeros(2, 8, 8), [])(torch.zeros(1, 8), torch.zeros(1, 1, dtype=torch.long),
                                                       torch.ones(1, 1), ["x"])


def test_adapter_bank_layers_match_reference(golden):
    from stageml_b200.adapter_bank import AdapterSpec, DynamicLoRALinear, OnTheFlyMergeLinear, StageMLAdapterBankLinear

    g = golden("adapter_bank")
    n = len(g["scaling"])
    ads = [AdapterSpec(f"adapter_{i}", torch.from_numpy(g[f"A{i}"]).to(DEV, BF), torch.from_numpy(g[f"B{i}"]).to(DEV, BF),
                       float(g["scaling"][i])) for i in range(n)]
    W = torch.from_numpy(g["W"]).to(DEV, BF)
    bias = torch.from_numpy(g["bias"]).to(DEV, BF)
    x = torch.from_numpy(g["x"]).to(DEV, BF)
    names = [f"adapter_{i}" for i in g["adapter_idx"]]
    A = np.stack([f64(a.A) for a in ads])
    B = np.stack([f64(a.B) for a in ads])
    ref = olora.dynamic_lora_linear(f64(x), f64(W), f64(bias), A, B, g["scaling"], g["adapter_idx"])
    for cls, gold in ((DynamicLoRALinear, "y_dyn"), (StageMLAdapterBankLinear, "y_bank"),
                      (OnTheFlyMergeLinear, "y_otf")):
        y = cls(W, ads, bias)(x, names)
        assert rel_l2(f64(y), ref) < 1e-2, cls.__name__
        assert rel_l2(f64(y), g[gold]) < 3e-2, cls.__name__


def test_cost_based_cache_matches_reference(golden):
    from stageml_b200.adapter_bank import AdapterSpec
    from stageml_b200.adapter_cache import StageMLCostBasedAdapterCache, choose_hot_adapters

    g = golden("adapter_cache")
    n = len(g["scaling"])
    ads = [AdapterSpec(f"adapter_{i}", torch.from_numpy(g[f"A{i}"]).to(DEV, BF), torch.from_numpy(g[f"B{i}"]).to(DEV, BF),
                       float(g["scaling"][i])) for i in range(n)]
    names = [f"adapter_{i}" for i in g["adapter_idx"]]
    counts = {}
    for nm in names:
        counts[nm] = counts.get(nm, 0) + 1
    cached, decisions = choose_hot_adapters(counts, ads, in_features=g["W"].shape[1], out_features=g["W"].shape[0],
                                            dtype=torch.float32, memory_budget_mb=float(g["budget_mb"]))
    assert [int(c.split("_")[1]) for c in cached] == list(g["cached"])
    assert [int(d.cached) for d in decisions] == list(g["decision_cached"])
    W = torch.from_numpy(g["W"]).to(DEV, BF)
    x = torch.from_numpy(g["x"]).to(DEV, BF)
    layer = StageMLCostBasedAdapterCache(W, ads, cached_adapter_names=cached)
    y = layer(x, names)
    A = np.stack([f64(a.A) for a in ads])
    B = np.stack([f64(a.B) for a in ads])
    ref = olora.cost_based_cache(f64(x), f64(W), None, A, B, g["scaling"], list(g["cached"]), g["adapter_idx"])
    assert rel_l2(f64(y), ref) < 1e-2
    assert rel_l2(f64(y), g["y"]) < 3e-2
    assert layer.cached_memory_bytes() == len(cached) * W.numel() * 2


def test_custom_op_registration_and_router_with_real_op():
    from stageml_b200.custom_op_registry import ensure_stageml_custom_op
    from stageml_b200.vllm_stage_router import StageMLTenantRouter, TenantKernel, route_fused_experts

    assert ensure_stageml_custom_op()
    g = torch.Generator().manual_seed(0)
    T, H, I, E = 40, 64, 64, 4
    h = torch.randn(T, H, generator=g).to(DEV, BF)
    gu = (torch.randn(E, 2 * I, H, generator=g) / 8).to(DEV, BF)
    dn = (torch.randn(E, H, I, generator=g) / 8).to(DEV, BF)
    ids = torch.randint(0, E, (T, 1), generator=g).to(DEV)
    w = torch.ones(T, 1, device=DEV)
    ten = torch.randint(0, 3, (T,), generator=g).to(DEV)
    fake_vllm = lambda hh, *a: torch.zeros((hh.shape[0], H), device=DEV, dtype=BF)
    router = StageMLTenantRouter({1: TenantKernel(1, 0, "stageml", "lib", "residual_moe")})
    out = route_fused_experts(hidden=h, gate_up=gu, down=dn, topk_weights=w, topk_ids=ids, tenant_ids=ten,
                              router=router, vllm_fused_experts=fake_vllm)
    full = torch.ops.stageml.residual_moe(h, gu, dn, w, ids)
    m = (ten == 1)
    assert torch.equal(out[~m], torch.zeros_like(out[~m]))
    ref = omoe.fallback_moe(f64(h), f64(gu), f64(dn), w.cpu().numpy(), ids.cpu().numpy())
    assert rel_l2(f64(out[m]), ref[m.cpu().numpy()]) < 1e-2
    assert rel_l2(f64(full), ref) < 1e-2
    # no host synchronisation: both backends on every token, the other side's weights zeroed
    masked = route_fused_experts(hidden=h, gate_up=gu, down=dn, topk_weights=w, topk_ids=ids, tenant_ids=ten,
                                 router=router, vllm_fused_experts=fake_vllm, split="masked")
    assert torch.equal(masked, out)
