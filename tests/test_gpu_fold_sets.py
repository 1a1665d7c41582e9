"""Folded and dynamic tenants in one MoE layer call (fold_slot / n_fold / down_group).

The permutation (every plan array bit-exact against the oracle's) and the layer
output (rel-L2 <= 1e-2 against the float64 oracle) through the C ABI, on the
shapes that take each device path: one-chunk ranks, tile pairs, the sort path
(more than 1024 keys), the decode-sized skinny GEMMs, shared experts and a
shared down projection. Then the callers that use it -- the residual-plan layer,
the request executor's batched mode and route_fused_experts(split="device") --
against the oracle, with no host read on their paths.
"""

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import moe as omoe
from oracle import permute as operm
from stageml_b200 import capi

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
BF = torch.bfloat16


@pytest.fixture(scope="module")
def lib():
    from stageml_b200._native import load_capi

    torch.cuda.init()
    return load_capi()


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def _case(T, H, I, E, k, nT, r, ns, n_fold, seed, shared_down=False):
    g = torch.Generator().manual_seed(seed)
    Et = E + ns
    x = torch.randn(T, H, generator=g).to(DEV, BF)
    gu = (torch.randn(Et + n_fold, 2 * I, H, generator=g) / H ** 0.5).to(DEV, BF)
    dn = (torch.randn(Et if shared_down else Et + n_fold, H, I, generator=g) / I ** 0.5).to(DEV, BF)
    lora = dict(lora_a13=(torch.randn(nT, Et, 2 * r, H, generator=g) / H ** 0.5).to(DEV, BF),
                lora_b13=(torch.randn(nT, Et, 2 * I, r, generator=g) / r ** 0.5).to(DEV, BF),
                lora_a2=(torch.randn(nT, Et, r, I, generator=g) / I ** 0.5).to(DEV, BF),
                lora_b2=(torch.randn(nT, Et, H, r, generator=g) / r ** 0.5).to(DEV, BF),
                lora_scale=torch.linspace(0.5, 2.0, nT).to(DEV))
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32).to(DEV)
    w = torch.softmax(torch.randn(T, k, generator=g), -1).to(DEV)
    ten = torch.randint(-1, nT, (T,), generator=g, dtype=torch.int32).to(DEV)
    # every folded set names one (tenant, expert); the rest of the map is dynamic
    fold = torch.full((nT, Et), -1, dtype=torch.int32)
    cells = torch.randperm(nT * Et, generator=g)[:n_fold]
    for s, c in enumerate(cells.tolist()):
        fold[c // Et, c % Et] = s
    down_group = None
    if shared_down:
        down_group = torch.tensor(list(range(Et)) + [int(c % Et) for c in cells.tolist()], dtype=torch.int32)
        down_group = down_group.to(DEV)
    return dict(x=x, gu=gu, dn=dn, ids=ids, w=w, ten=ten, fold=fold.to(DEV), down_group=down_group, **lora)


def _oracle(c, ns):
    return omoe.moe_forward(f64(c["x"]), f64(c["gu"]), f64(c["dn"]), c["ids"].cpu().numpy(), c["w"].cpu().numpy(),
                            tenant_ids=c["ten"].cpu().numpy(), n_shared=ns, lora_a13=f64(c["lora_a13"]),
                            lora_b13=f64(c["lora_b13"]), lora_a2=f64(c["lora_a2"]), lora_b2=f64(c["lora_b2"]),
                            lora_scale=c["lora_scale"].cpu().numpy(), fold_slot=c["fold"].cpu().numpy(),
                            down_group=None if c["down_group"] is None else c["down_group"].cpu().numpy())


CASES = [
    dict(T=300, H=256, I=384, E=4, k=2, nT=3, r=16, ns=0, n_fold=3),                    # one chunk of ranks
    dict(T=2048, H=256, I=256, E=4, k=2, nT=5, r=16, ns=0, n_fold=6),                   # tile pairs
    dict(T=1500, H=128, I=128, E=8, k=2, nT=140, r=8, ns=0, n_fold=40),                 # > 1024 keys: sort path
    dict(T=3, H=256, I=256, E=4, k=2, nT=3, r=16, ns=0, n_fold=4),                      # skinny GEMMs
    dict(T=400, H=128, I=192, E=6, k=2, nT=4, r=16, ns=2, n_fold=5),                    # shared experts
    dict(T=700, H=256, I=256, E=4, k=2, nT=4, r=16, ns=0, n_fold=5, shared_down=True),  # shared down weights
]


@pytest.mark.parametrize("case", CASES)
def test_fold_slots_through_c_abi(lib, case):
    c = _case(seed=11, **{k: v for k, v in case.items()})
    T, H, I, E, k, nT, r, ns, nf = (case[n] for n in ("T", "H", "I", "E", "k", "nT", "r", "ns", "n_fold"))
    Et = E + ns
    out = torch.empty(T, H, device=DEV, dtype=BF)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    P = T * (k + ns)
    G = Et + nf
    cap = lib.stageml_plan_rows_cap(P, G)
    bufs = {n: torch.empty(cap, dtype=torch.int32, device=DEV) for n in ("row_token", "row_tenant", "row_pair")}
    bufs["row_weight"] = torch.empty(cap, dtype=torch.float32, device=DEV)
    bufs["pair_row"] = torch.empty(P, dtype=torch.int32, device=DEV)
    bufs["tile_group"] = torch.empty(cap // 128, dtype=torch.int32, device=DEV)
    bufs["group_offsets"] = torch.empty(G + 1, dtype=torch.int32, device=DEV)
    bufs["group_counts"] = torch.empty(G, dtype=torch.int32, device=DEV)
    bufs["num_tiles"] = torch.empty(1, dtype=torch.int32, device=DEV)
    plan = capi.MoePlan(**{n: t.data_ptr() for n, t in bufs.items()}, rows_cap=cap)
    a = capi.MoeArgs(T=T, H=H, I=I, E=E, k=k, n_shared=ns, act_dtype=capi.BF16, weight_dtype=capi.BF16,
                     x=c["x"].data_ptr(), topk_ids=c["ids"].data_ptr(), ids_dtype=capi.I32,
                     topk_weights=c["w"].data_ptr(), weights_dtype=capi.F32, tenant_ids=c["ten"].data_ptr(),
                     n_tenants=nT, rank=r, gate_up=c["gu"].data_ptr(), down=c["dn"].data_ptr(),
                     lora_a13=c["lora_a13"].data_ptr(), lora_b13=c["lora_b13"].data_ptr(),
                     lora_a2=c["lora_a2"].data_ptr(), lora_b2=c["lora_b2"].data_ptr(),
                     lora_scale=c["lora_scale"].data_ptr(), out=out.data_ptr(), status=status.data_ptr(),
                     plan_out=ctypes.addressof(plan), fold_slot=c["fold"].data_ptr(), n_fold=nf,
                     down_group=None if c["down_group"] is None else c["down_group"].data_ptr())
    need = lib.stageml_moe_workspace_bytes(ctypes.byref(a))
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    capi.check(lib, lib.stageml_moe_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), need,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "moe fold")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    pref = operm.permute(c["ids"].cpu().numpy(), c["w"].cpu().numpy(), c["ten"].cpu().numpy(), Et, ns, nT,
                         fold_slot=c["fold"].cpu().numpy(), n_fold=nf)
    nt = int(bufs["num_tiles"].item())
    assert nt == pref["num_tiles"]
    for n in ("row_token", "row_tenant", "row_pair"):
        np.testing.assert_array_equal(bufs[n][: nt * 128].cpu().numpy(), pref[n], err_msg=n)
    np.testing.assert_array_equal(bufs["row_weight"][: nt * 128].cpu().numpy(), pref["row_weight"])
    np.testing.assert_array_equal(bufs["pair_row"].cpu().numpy(), pref["pair_row"])
    np.testing.assert_array_equal(bufs["tile_group"][:nt].cpu().numpy(), pref["tile_group"])
    np.testing.assert_array_equal(bufs["group_offsets"].cpu().numpy(), pref["group_offsets"])
    np.testing.assert_array_equal(bufs["group_counts"].cpu().numpy(), pref["group_counts"])
    assert rel_l2(f64(out), _oracle(c, ns)) < 1e-2
    # the torch op gives the same bits
    import stageml_b200.ops as ops

    y = ops.moe_forward(c["x"], c["gu"], c["dn"], topk_ids=c["ids"], topk_weights=c["w"], n_shared=ns,
                        tenant_ids=c["ten"], n_tenants=nT, rank=r, lora_a13=c["lora_a13"], lora_b13=c["lora_b13"],
                        lora_a2=c["lora_a2"], lora_b2=c["lora_b2"], lora_scale=c["lora_scale"], fold_slot=c["fold"],
                        n_fold=nf, down_group=c["down_group"])
    assert torch.equal(y, out)


def test_fold_slot_out_of_range_is_reported_and_dropped():
    import stageml_b200.ops as ops

    c = _case(T=200, H=128, I=128, E=4, k=2, nT=3, r=16, ns=0, n_fold=2, seed=3)
    ten = c["ten"].cpu().numpy()
    a = int(ten[ten >= 0][0])
    e = int(c["ids"][int(np.nonzero(ten == a)[0][0]), 0])
    c["fold"][a, e] = 2  # == n_fold: out of range
    kw = dict(topk_ids=c["ids"], topk_weights=c["w"], tenant_ids=c["ten"], n_tenants=3, rank=16,
              lora_a13=c["lora_a13"], lora_b13=c["lora_b13"], lora_a2=c["lora_a2"], lora_b2=c["lora_b2"],
              lora_scale=c["lora_scale"], fold_slot=c["fold"], n_fold=2)
    y = ops.moe_forward(c["x"], c["gu"], c["dn"], **kw)
    assert ops.take_status(y) == 110  # STAGEML_DEV_BAD_INDEX
    # the dropped pairs contribute nothing: the oracle with their routing weight zeroed
    ids = c["ids"].cpu().numpy()
    w = c["w"].cpu().numpy().copy()
    w[(ten == a)[:, None] & (ids == e)] = 0.0
    fold_ok = c["fold"].clone()
    fold_ok[a, e] = -1
    ref = omoe.moe_forward(f64(c["x"]), f64(c["gu"]), f64(c["dn"]), ids, w, tenant_ids=ten,
                           lora_a13=f64(c["lora_a13"]), lora_b13=f64(c["lora_b13"]), lora_a2=f64(c["lora_a2"]),
                           lora_b2=f64(c["lora_b2"]), lora_scale=c["lora_scale"].cpu().numpy(),
                           fold_slot=fold_ok.cpu().numpy())
    assert rel_l2(f64(y), ref) < 1e-2
    with pytest.raises(RuntimeError, match="E4M3|fold"):
        q = c["gu"].to(torch.float8_e4m3fn)
        ops.moe_forward(c["x"], q, c["dn"].to(torch.float8_e4m3fn), gate_up_scale=torch.ones(4, 256, device=DEV),
                        down_scale=torch.ones(4, 128, device=DEV), **kw)


def _w1_adapters(E, I, H, r, n, seed):
    from stageml_b200.moe_lora_layers import MoEAdapterSpec

    g = torch.Generator().manual_seed(seed)
    return [MoEAdapterSpec(f"adapter_{i}", (torch.randn(E, r, H, generator=g) / H ** 0.5).to(DEV, BF),
                           (torch.randn(E, I, r, generator=g) / r ** 0.5).to(DEV, BF), 1.0 + 0.5 * i)
            for i in range(n)]


def _oracle_w1(x, gate_up, down, ids, w, ten, ads, folded: dict, dynamic: bool = True):
    """Oracle of a w1-adapter layer where adapter a is folded into the experts folded[a]
    (and, with ``dynamic``, applied as LoRA on its other experts)."""
    E, I2, H = gate_up.shape
    I = I2 // 2
    n = len(ads)
    r = max(a.rank for a in ads)
    a13 = np.zeros((n, E, 2 * r, H))
    b13 = np.zeros((n, E, I2, r))
    for i, a in enumerate(ads):
        a13[i, :, : a.rank] = f64(a.A)
        b13[i, :, :I, : a.rank] = f64(a.B)
    sc = np.array([a.scaling for a in ads])
    gu, fold = [f64(gate_up)], np.full((n, E), -1)
    dgroup = list(range(E))
    for a, ex in sorted(folded.items()):
        for e in ex:
            fold[a, e] = len(dgroup) - E
            g = f64(gate_up[e]).copy()
            g[:I] += sc[a] * b13[a, e, :I, : ads[a].rank] @ a13[a, e, : ads[a].rank]
            gu.append(g[None])
            dgroup.append(e)
    lora = dict(lora_a13=a13, lora_b13=b13, lora_scale=sc) if dynamic else {}
    return omoe.moe_forward(f64(x), np.concatenate(gu), f64(down), ids.cpu().numpy(), w.cpu().numpy(),
                            tenant_ids=ten.cpu().numpy(), fold_slot=fold, down_group=np.array(dgroup), **lora)


def test_planned_layer_against_oracle():
    from stageml_b200 import ops
    from stageml_b200.residual_plan import PlannedMoELayer, read_residual_plan

    torch.manual_seed(0)
    T, H, I, E, k, nA, r = 700, 256, 384, 6, 2, 4, 16
    x = torch.randn(T, H, device=DEV).to(BF)
    gate_up = (torch.randn(E, 2 * I, H, device=DEV) * H ** -0.5).to(BF)
    down = (torch.randn(E, H, I, device=DEV) * I ** -0.5).to(BF)
    ids = torch.stack([torch.randperm(E, device=DEV)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, device=DEV), -1)
    ads = _w1_adapters(E, I, H, r, nA, 1)
    entry = lambda a, e, kind: {"adapter": a, "expert": e, "kind": kind, "rank": r, "memory_bytes": 0,
                                "estimated_latency_cost": 0.0, "epsilon": 0.0, "reason": ""}
    plan = read_residual_plan({"plans": [entry("adapter_1", "all", "materialized_residual"),
                                         entry("adapter_2", 1, "materialized_residual"),
                                         entry("adapter_2", 4, "materialized_residual"),
                                         entry("adapter_0", "all", "non_materializing_fusion"),
                                         entry("adapter_3", "all", "fallback")]})
    layer = PlannedMoELayer(gate_up, down, ads, plan)
    assert layer.sets.n_fold == E + 2
    ten = torch.randint(-1, nA, (T,), device=DEV, dtype=torch.int32)
    y = layer(x, ids, w, ten)
    assert ops.take_status(x) == 0
    ref = _oracle_w1(x, gate_up, down, ids, w, ten, ads, {1: list(range(E)), 2: [1, 4]})
    assert rel_l2(f64(y), ref) < 1e-2


def test_executor_batched_mode_runs_materialized_adapters_folded():
    from stageml_b200.executor import RequestExecutor, make_workload_plan

    torch.manual_seed(1)
    T, H, I, E, k, nA, r = 512, 256, 384, 6, 2, 5, 16
    hidden = torch.randn(T, H, device=DEV).to(BF)
    gate_up = (torch.randn(E, 2 * I, H, device=DEV) * H ** -0.5).to(BF)
    down = (torch.randn(E, H, I, device=DEV) * I ** -0.5).to(BF)
    ids = torch.stack([torch.randperm(E, device=DEV)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, device=DEV), -1)
    ads = _w1_adapters(E, I, H, r, nA, 2)
    plan = make_workload_plan(num_requests=30, num_tenants=9, num_adapters=nA, tokens_available=T,
                              tokens_per_request=24, distribution="zipf", zipf_alpha=1.1, burst_size=1,
                              materialization_policy="top_k", materialize_top_k=2, materialize_min_requests=1,
                              memory_budget_mb=0, memory_per_adapter_bytes=0, seed=3)
    assert plan.materialized_adapter_ids
    ex = RequestExecutor(gate_up, down, ads, plan.materialized_adapter_ids)
    y, off = ex.run_batched(plan, hidden, ids, w)
    rows = torch.cat([torch.arange(q.start, q.end) for q in plan.requests]).to(DEV)
    ten = torch.cat([torch.full((q.end - q.start,), q.adapter_id, dtype=torch.int32) for q in plan.requests]).to(DEV)
    ref = _oracle_w1(hidden[rows], gate_up, down, ids[rows], w[rows], ten, ads,
                     {a: list(range(E)) for a in plan.materialized_adapter_ids})
    assert rel_l2(f64(y), ref) < 1e-2
    # a materialized adapter's rows equal its bta_one rows (same folded weights, same sums)
    for q, req in enumerate(plan.requests):
        if req.adapter_id in plan.materialized_adapter_ids:
            bta = ex.bta_one(hidden[req.start:req.end], ids[req.start:req.end], w[req.start:req.end], req.adapter_id)
            assert rel_l2(f64(y[off[q]:off[q + 1]]), f64(bta)) < 1e-2
            break


def test_route_fused_experts_device_split_against_oracle():
    from stageml_b200.folded_sets import fold_w1_sets
    from stageml_b200.vllm_stage_router import StageMLTenantRouter, TenantKernel, route_fused_experts

    torch.manual_seed(2)
    T, H, I, E, k, nA, r = 300, 128, 256, 4, 2, 4, 16
    x = torch.randn(T, H, device=DEV).to(BF)
    gate_up = (torch.randn(E, 2 * I, H, device=DEV) * H ** -0.5).to(BF)
    down = (torch.randn(E, H, I, device=DEV) * I ** -0.5).to(BF)
    ids = torch.stack([torch.randperm(E, device=DEV)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, device=DEV), -1)
    ads = _w1_adapters(E, I, H, r, nA, 3)
    sets = fold_w1_sets(gate_up, down, ads, [(1, list(range(E))), (2, [0, 3])])
    router = StageMLTenantRouter({t: TenantKernel(t, t, "stageml_b200", "folded", "residual_moe") for t in (1, 2)})
    ten = torch.randint(-1, nA, (T,), device=DEV, dtype=torch.int32)
    never = lambda *a, **kw: (_ for _ in ()).throw(AssertionError("vLLM must not be called"))
    y = route_fused_experts(hidden=x, gate_up=gate_up, down=down, topk_weights=w, topk_ids=ids, tenant_ids=ten,
                            router=router, vllm_fused_experts=never, split="device", weight_sets=sets)
    # tenants 1 and 2 on their folded sets (tenant 2 only on experts 0 and 3), every other
    # (token, expert) on the base experts; no dynamic LoRA in this form
    routed = torch.where((ten == 1) | (ten == 2), ten, torch.full_like(ten, -1))
    ref = _oracle_w1(x, gate_up, down, ids, w, routed, ads, {1: list(range(E)), 2: [0, 3]}, dynamic=False)
    assert rel_l2(f64(y), ref) < 1e-2
    base = route_fused_experts(hidden=x, gate_up=gate_up, down=down, topk_weights=w, topk_ids=ids, tenant_ids=ten,
                               router=router, vllm_fused_experts=never, split="device")
    ref0 = omoe.fallback_moe(f64(x), f64(gate_up), f64(down), w.cpu().numpy(), ids.cpu().numpy())
    assert rel_l2(f64(base), ref0) < 1e-2
