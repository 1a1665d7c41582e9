"""The dense and fine-grained configurations at their benchmark shapes, against the oracle.

- Multi-tenant LoRA bank: 256 tokens x 4096 -> 4096 bf16, 64 rank-16 adapters (scale 2),
  Zipf(1.1) adapter ids, the 8 most requested adapters folded at stage 0
  (StageMLCostBasedAdapterCache + choose_hot_adapters, stageml/adapter_cache.py:37-140).
- LLaMA-7B block projections, fp16: 16 x 128 tokens, q/k/v/o 4096x4096 through
  DynamicLoRALinear (stageml/adapter_bank.py:58-69) and the SwiGLU MLP
  4096 -> 11008 -> 4096 as a one-expert MoE layer, rank-16 LoRA on all 7 projections
  for 16 tenants (one per sequence); checked on two tokens of every sequence.
- Fine-grained FP8 MoE-LoRA layer: 8192 tokens, H=2048, I=1408, 64 routed experts top-6
  plus 2 shared, e4m3 weights with per-output-channel scales, rank-8 LoRA for 128 Zipf
  tenants; e4m3 codes bit-exact on sampled experts, layer output checked on sampled
  tokens over all their experts (oracle on the dequantised weights).
Bars: ids and codes bit-exact; 16-bit outputs rel-L2 <= 1e-2 against the float64 oracle.
"""

import numpy as np
import pytest
import torch

from conftest import oracle_moe_tokens, rel_l2
from oracle import lora as olora
from oracle import numerics
from oracle.route import topk_from_logits

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL16 = 1e-2


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_adapter_bank_at_benchmark_shape():
    from stageml_b200 import workloads as wl
    from stageml_b200.adapter_bank import AdapterSpec
    from stageml_b200.adapter_cache import StageMLCostBasedAdapterCache, choose_hot_adapters

    w = wl.make_adapter_bank(seed=0, device=DEV, gen_device="cpu")
    n, dim = w["A"].shape[0], w["W"].shape[0]
    assert (w["x"].shape, n, w["A"].shape[1]) == ((256, 4096), 64, 16)
    ads = [AdapterSpec(f"adapter_{i}", w["A"][i], w["B"][i], w["scale"]) for i in range(n)]
    names = [f"adapter_{i}" for i in w["adapter_ids"]]
    counts = {}
    for nm in names:
        counts[nm] = counts.get(nm, 0) + 1
    budget_mb = 8 * dim * dim * 2 / 2 ** 20  # eight folded bf16 matrices
    cached, _ = choose_hot_adapters(counts, ads, in_features=dim, out_features=dim, dtype=torch.bfloat16,
                                    memory_budget_mb=budget_mb)
    ref_cached = olora.choose_hot_adapters(counts, [a.name for a in ads], in_features=dim, out_features=dim,
                                           bytes_per_weight=2, memory_budget_mb=budget_mb)
    assert cached == ref_cached and len(cached) == 8
    assert sorted(int(c.split("_")[1]) for c in cached) == sorted(w["folded"])
    layer = StageMLCostBasedAdapterCache(w["W"], ads, cached_adapter_names=cached)
    y = layer(w["x"], names)
    torch.cuda.synchronize()
    A = f64(w["A"])
    B = f64(w["B"])
    ref = olora.cost_based_cache(f64(w["x"]), f64(w["W"]), None, A, B, np.full(n, w["scale"]),
                                 [int(c.split("_")[1]) for c in cached], np.asarray(w["adapter_ids"]))
    assert rel_l2(f64(y), ref) < TOL16
    # the folded rows really ran on folded weights: the same layer with nothing cached agrees
    y_dyn = StageMLCostBasedAdapterCache(w["W"], ads, cached_adapter_names=[])(w["x"], names)
    assert rel_l2(f64(y_dyn), ref) < TOL16


def test_llama_block_projections_at_benchmark_shape():
    import stageml_b200.ops as ops
    from stageml_b200 import workloads as wl
    from stageml_b200.adapter_bank import AdapterSpec, DynamicLoRALinear
    from oracle import moe as omoe

    blk = wl.make_llama_block(seed=0, device=DEV)
    P, ten = blk["proj"], blk["row_tenant"]
    M, nT, r = blk["x"].shape[0], 16, 16
    assert M == 2048 and blk["x"].dtype == torch.float16
    names = [f"tenant_{t}" for t in ten.tolist()]
    sel = np.array([s * 128 + j for s in range(16) for j in (5, 127)])
    ten_np = ten.cpu().numpy()
    scale = np.full(nT, blk["scale"])
    for p in "qkvo":
        ads = [AdapterSpec(f"tenant_{a}", P[p]["A"][a], P[p]["B"][a], blk["scale"]) for a in range(nT)]
        x = blk["x_o"] if p == "o" else blk["x"]
        y = DynamicLoRALinear(P[p]["W"], ads)(x, names)
        ref = olora.dynamic_lora_linear(f64(x[sel]), f64(P[p]["W"]), None, f64(P[p]["A"]), f64(P[p]["B"]), scale,
                                        ten_np[sel])
        assert rel_l2(f64(y[sel]), ref) < TOL16, p
    # SwiGLU MLP: a one-expert MoE layer, gate_up = [W_gate; W_up], LoRA A13 = [A_gate; A_up]
    gu = torch.cat([P["gate"]["W"], P["up"]["W"]], 0)[None].contiguous()
    dn = P["down"]["W"][None].contiguous()
    a13 = torch.cat([P["gate"]["A"], P["up"]["A"]], 1)[:, None].contiguous()
    b13 = torch.cat([P["gate"]["B"], P["up"]["B"]], 1)[:, None].contiguous()
    a2, b2 = P["down"]["A"][:, None].contiguous(), P["down"]["B"][:, None].contiguous()
    ids = torch.zeros(M, 1, dtype=torch.int32, device=DEV)
    ones = torch.ones(M, 1, dtype=torch.float32, device=DEV)
    sc = torch.full((nT,), blk["scale"], dtype=torch.float32, device=DEV)
    y = ops.moe_forward(blk["x"], gu, dn, topk_ids=ids, topk_weights=ones, tenant_ids=ten, n_tenants=nT, rank=r,
                        lora_a13=a13, lora_b13=b13, lora_a2=a2, lora_b2=b2, lora_scale=sc)
    assert ops.take_status(y) == 0
    ref = omoe.moe_forward(f64(blk["x"][sel]), f64(gu), f64(dn), np.zeros((sel.size, 1), np.int64),
                           np.ones((sel.size, 1)), tenant_ids=ten_np[sel], lora_a13=f64(a13), lora_b13=f64(b13),
                           lora_a2=f64(a2), lora_b2=f64(b2), lora_scale=scale)
    assert rel_l2(f64(y[sel]), ref) < TOL16


@pytest.fixture(scope="module")
def fine_grained():
    import stageml_b200.ops as ops
    from stageml_b200.workloads import MOE_CONFIGS, make_moe_workload

    cfg = MOE_CONFIGS["fine_grained_fp8_moe_lora"]
    w16 = make_moe_workload(cfg.__class__(**dict(cfg.__dict__, weight_dtype="bf16")), device=DEV, seed=0)
    w = dict(w16)
    for n in ("gate_up", "down"):  # what the e4m3 workload does with the same draws
        q, s = ops.quantize_e4m3_rows(w16[n].reshape(-1, w16[n].shape[-1]))
        w[n] = q.view(w16[n].shape)
        w[n + "_scale"] = s.view(w16[n].shape[:-1]).contiguous()
    return cfg, w16, w, ops


def test_fine_grained_fp8_codes_bit_exact(fine_grained):
    cfg, w16, w, ops = fine_grained
    for n in ("gate_up", "down"):
        for e in (0, 37, cfg.E, cfg.E_tot - 1):  # routed and shared experts
            q, s = numerics.quantize_e4m3_rows(w16[n][e].float().cpu().numpy())
            np.testing.assert_array_equal(w[n][e].view(torch.uint8).cpu().numpy(), q)
            np.testing.assert_array_equal(w[n + "_scale"][e].cpu().numpy(), s)


def test_fine_grained_fp8_layer_at_benchmark_shape(fine_grained):
    cfg, w16, w, ops = fine_grained
    assert (cfg.T, cfg.H, cfg.I, cfg.E, cfg.k, cfg.n_shared, cfg.rank, cfg.n_tenants) == (
        8192, 2048, 1408, 64, 6, 2, 8, 128)
    y = ops.moe_forward(w["x"], w["gate_up"], w["down"], router_w=w["router_w"], k=cfg.k, n_shared=cfg.n_shared,
                        tenant_ids=w["tenant_ids"], n_tenants=cfg.n_tenants, rank=cfg.bank_rank,
                        lora_a13=w["lora_a13"], lora_b13=w["lora_b13"], lora_a2=w["lora_a2"], lora_b2=w["lora_b2"],
                        lora_scale=w["lora_scale"], gate_up_scale=w["gate_up_scale"], down_scale=w["down_scale"])
    assert ops.take_status(y) == 0
    ids, wts, logits = ops.route_topk(w["x"], w["router_w"], cfg.k, True)
    ref_ids, _ = topk_from_logits(logits.cpu().numpy(), cfg.k, True)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
    ids, wts = ids.cpu().numpy(), wts.cpu().numpy()
    ten = w["tenant_ids"].cpu().numpy()
    # the most frequent tenant, a mid one and the rarest ones seen (the last rows of their experts' segments)
    order = np.argsort(ten, kind="stable")
    sel = np.unique(np.concatenate([order[:4], order[cfg.T // 2:cfg.T // 2 + 2], order[-6:]]))
    f32 = lambda t: t.float().cpu().numpy()

    def expert(e):
        g = numerics.dequantize_e4m3_rows(w["gate_up"][e].view(torch.uint8).cpu().numpy(),
                                          w["gate_up_scale"][e].cpu().numpy())
        d = numerics.dequantize_e4m3_rows(w["down"][e].view(torch.uint8).cpu().numpy(),
                                          w["down_scale"][e].cpu().numpy())
        return g, d

    lora = lambda e: tuple(f32(w[n][:, e:e + 1]) for n in ("lora_a13", "lora_b13", "lora_a2", "lora_b2"))
    ref = oracle_moe_tokens(np.arange(sel.size), ids[sel], wts[sel], ten[sel], f32(w["x"])[sel], expert, lora,
                            f32(w["lora_scale"]), n_routed=cfg.E, n_shared=cfg.n_shared)
    assert rel_l2(f32(y)[sel], ref) < TOL16
