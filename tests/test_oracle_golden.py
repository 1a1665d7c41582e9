"""The CPU oracle against golden vectors produced by running the reference (tests/golden/make_golden.py).

This pins the restatement: every function the GPU parity tests trust is first
checked here against the reference's own outputs (fp32, tolerance 1e-5 as the
reference's tests use).
"""

import numpy as np

from conftest import load_golden, rel_l2
from oracle import lora, moe, permute, route

TOL = 1e-5


def test_moe_lora_layers_dynamic_and_materialized():
    g = load_golden("moe_lora_layers")
    n = len(g["scaling"])
    A = [g[f"A{i}"] for i in range(n)]
    B = [g[f"B{i}"] for i in range(n)]
    aidx = g["adapter_idx"]
    T, E = g["x"].shape[0], g["W"].shape[0]
    r_max = max(a.shape[1] for a in A)
    # pad ranks into banks [n, E, r, in] / [n, E, out, r] -- zero rank columns add nothing
    a_bank = np.zeros((n, E, r_max, g["x"].shape[1]))
    b_bank = np.zeros((n, E, g["W"].shape[1], r_max))
    for i in range(n):
        a_bank[i, :, : A[i].shape[1]] = A[i]
        b_bank[i, :, :, : B[i].shape[2]] = B[i]
    y = moe.moe_linear(g["x"], g["W"], g["ids"], g["rw"], tenant_ids=aidx, lora_a=a_bank, lora_b=b_bank,
                       lora_scale=g["scaling"])
    assert rel_l2(y, g["y_dyn"]) < TOL
    merged = np.stack([lora.lora_fold(g["W"][e], A[i][e], B[i][e], g["scaling"][i]) for i in range(n)
                       for e in range(E)]).reshape(n, E, *g["W"].shape[1:])
    assert rel_l2(merged, g["merged"]) < TOL
    y_mat = moe.moe_linear(g["x"], None, g["ids"], g["rw"], tenant_ids=aidx, merged=merged)
    assert rel_l2(y_mat, g["y_mat"]) < TOL


def test_adapter_bank_layers():
    g = load_golden("adapter_bank")
    n = len(g["scaling"])
    A = np.stack([g[f"A{i}"] for i in range(n)])
    B = np.stack([g[f"B{i}"] for i in range(n)])
    y = lora.dynamic_lora_linear(g["x"], g["W"], g["bias"], A, B, g["scaling"], g["adapter_idx"])
    assert rel_l2(y, g["y_dyn"]) < TOL
    merged = np.stack([lora.lora_fold(g["W"], A[i], B[i], g["scaling"][i]) for i in range(n)])
    yb = lora.adapter_bank_linear(g["x"], merged, g["bias"], g["adapter_idx"])
    assert rel_l2(yb, g["y_bank"]) < TOL
    assert rel_l2(yb, g["y_otf"]) < TOL


def test_cost_based_cache_and_policy():
    g = load_golden("adapter_cache")
    n = len(g["scaling"])
    A = np.stack([g[f"A{i}"] for i in range(n)])
    B = np.stack([g[f"B{i}"] for i in range(n)])
    counts = {}
    for a in g["adapter_idx"]:
        counts[f"adapter_{a}"] = counts.get(f"adapter_{a}", 0) + 1
    cached = lora.choose_hot_adapters(counts, [f"adapter_{i}" for i in range(n)], in_features=g["W"].shape[1],
                                      out_features=g["W"].shape[0], bytes_per_weight=4,
                                      memory_budget_mb=float(g["budget_mb"]))
    assert [int(c.split("_")[1]) for c in cached] == list(g["cached"])
    y = lora.cost_based_cache(g["x"], g["W"], None, A, B, g["scaling"], list(g["cached"]), g["adapter_idx"])
    assert rel_l2(y, g["y"]) < TOL


def test_fold_known_answer_and_random():
    g = load_golden("fold")
    out = lora.lora_fold(g["known_W"], g["known_A"], g["known_B"], float(g["known_scale"]))
    np.testing.assert_array_equal(out, g["known_out"])
    np.testing.assert_array_equal(out, np.ones((3, 4)))
    assert rel_l2(lora.lora_fold(g["W"], g["A"], g["B"], float(g["scale"])), g["out"]) < TOL


def test_fallback_moe():
    g = load_golden("fallback_moe")
    y = moe.fallback_moe(g["hidden"], g["gate_up"], g["down"], g["topk_weights"], g["topk_ids"])
    assert rel_l2(y, g["out"]) < TOL


def test_request_executor_dynamic_and_bta():
    g = load_golden("request_executor")
    E, r, H = g["A0"].shape
    I = g["gate_up"].shape[1] // 2
    for i in range(2):
        a13 = np.zeros((1, E, 2 * r, H))
        b13 = np.zeros((1, E, 2 * I, r))
        a13[0, :, :r] = g[f"A{i}"]
        b13[0, :, :I] = g[f"B{i}"]
        y = moe.moe_forward(g["x"], g["gate_up"], g["down"], g["topk_ids"], g["topk_weights"],
                            tenant_ids=np.zeros(g["x"].shape[0], int), lora_a13=a13, lora_b13=b13,
                            lora_scale=np.array([g["scaling"][i]]))
        assert rel_l2(y, g[f"dyn{i}"]) < TOL
        assert rel_l2(y, g[f"bta{i}"]) < TOL  # folding w1 (bta_one) does not change the result
    # the folded gate_up of adapter 0 = [w1 + s B A ; w3]
    w1 = g["gate_up"][:, :I]
    fold = np.stack([lora.lora_fold(w1[e], g["A0"][e], g["B0"][e], g["scaling"][0]) for e in range(E)])
    assert rel_l2(fold, g["residual_gate_up0"][:, :I]) < TOL
    np.testing.assert_array_equal(g["residual_gate_up0"][:, I:], g["gate_up"][:, I:])


def test_router_matches_make_routing():
    g = load_golden("routing")
    ids, w, _ = route.route_topk(g["hidden"], g["gate_w"], int(g["k"]))
    np.testing.assert_array_equal(ids, g["ids"])
    assert rel_l2(w, g["weights"]) < TOL


def test_single_lora_rewrite_and_fold():
    g = load_golden("single_lora")
    assert int(g["rewrites"]) >= 1
    y = lora.single_lora(g["x"], g["W"], g["A"], g["B"], float(g["scale"]))
    assert rel_l2(y, g["y"]) < TOL
    folded = lora.lora_fold(g["W"], g["A"], g["B"], float(g["scale"]), layout=1)
    assert rel_l2(g["x"].astype(np.float64) @ folded, g["y_residual"]) < TOL


def test_tenant_sampler_matches_reference():
    from stageml_b200.workloads import sample_tenants

    g = load_golden("tenants")
    for dist in ("uniform", "zipf", "round_robin", "bursty"):
        assert sample_tenants(50, 16, dist, 1.1, burst=3, seed=11) == list(g[dist])


def test_permutation_is_stable_sort_by_expert_then_tenant():
    rng = np.random.default_rng(0)
    T, k, E, nT = 300, 2, 6, 4
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    ten = rng.integers(-1, nT, T)
    w = rng.random((T, k)).astype(np.float32)
    p = permute.permute(ids, w, ten, E, 0, nT)
    assert p["dropped"] == 0
    rows = p["row_pair"][p["row_pair"] >= 0]
    key = ids.reshape(-1) * (nT + 1) + (np.repeat(ten, k) + 1)
    np.testing.assert_array_equal(rows, np.lexsort((np.arange(T * k), key)))
    # segments are padded to 128 and contiguous per expert
    assert np.all(p["group_offsets"] % 128 == 0)
    for e in range(E):
        seg = p["row_pair"][p["group_offsets"][e]: p["group_offsets"][e] + p["group_counts"][e]]
        assert np.all(ids.reshape(-1)[seg] == e)
    # inverse
    np.testing.assert_array_equal(p["row_pair"][p["pair_row"]], np.arange(T * k))


def test_torch_executor_restatement_matches_reference_request_executor(golden):
    """The torch restatement of RequestExecutor.dynamic_one (the benchmark's timed CPU baseline)
    against the reference executor's own outputs, and against the numpy oracle with LoRA on
    w1, w3, w2, per-token tenants and a shared expert."""
    import torch

    from oracle import moe as omoe
    from oracle.torch_executor import dynamic_executor

    g = golden("request_executor")
    t = lambda n: torch.from_numpy(np.asarray(g[n], dtype=np.float32))
    E, I2, H = g["gate_up"].shape
    I = I2 // 2
    for a in (0, 1):
        A, B = t(f"A{a}"), t(f"B{a}")
        r = A.shape[1]
        a13 = torch.zeros(1, E, 2 * r, H)
        b13 = torch.zeros(1, E, I2, r)
        a13[0, :, :r] = A
        b13[0, :, :I] = B
        T = g["x"].shape[0]
        y = dynamic_executor(t("x"), t("gate_up"), t("down"), torch.from_numpy(g["topk_ids"]), t("topk_weights"),
                             torch.zeros(T, dtype=torch.int32), lora_a13=a13, lora_b13=b13,
                             lora_scale=torch.tensor([float(g["scaling"][a])]))
        assert rel_l2(y.numpy(), g[f"dyn{a}"]) < 1e-5
    rng = np.random.default_rng(3)
    T, H, I, E, k, nT, r, ns = 30, 16, 12, 4, 2, 3, 4, 1
    Et = E + ns
    arr = lambda *s: rng.normal(size=s).astype(np.float32) / 3
    x, gu, dn = arr(T, H), arr(Et, 2 * I, H), arr(Et, H, I)
    lo = dict(lora_a13=arr(nT, Et, 2 * r, H), lora_b13=arr(nT, Et, 2 * I, r), lora_a2=arr(nT, Et, r, I),
              lora_b2=arr(nT, Et, H, r), lora_scale=np.array([0.5, 1.0, 2.0], dtype=np.float32))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    w = rng.random((T, k)).astype(np.float32)
    ten = rng.integers(-1, nT, T).astype(np.int32)
    ref = omoe.moe_forward(x, gu, dn, ids, w, tenant_ids=ten, n_shared=ns, **lo)
    T_ = torch.from_numpy
    y = dynamic_executor(T_(x), T_(gu), T_(dn), T_(ids), T_(w), T_(ten), n_shared=ns,
                         **{n: T_(v) for n, v in lo.items()})
    assert rel_l2(y.numpy(), ref) < 1e-5
