"""GPU parity of every op of the residual path against the CPU oracle (run with -m gpu).

Tolerances: integer / index outputs (routing ids, permutation, e4m3 codes) are
compared bit for bit; bf16 / fp16 outputs within rel-L2 1e-2 of the oracle
evaluated in float64 on the same (16-bit) inputs; fp32 paths within 1e-5.
"""

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import lora as olora
from oracle import moe as omoe
from oracle import numerics, permute as operm, route as oroute

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
TOL32 = 1e-5
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ops():
    import stageml_b200.ops as o

    return o


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def rand(shape, scale=1.0, dtype=torch.bfloat16, seed=None, device=DEV):
    g = torch.Generator(device="cpu").manual_seed(seed if seed is not None else hash(shape) % 2 ** 31)
    return (torch.randn(*shape, generator=g) * scale).to(device=device, dtype=dtype)


def check_status(ops, expect=0):
    assert ops.take_status(torch.empty(1, device=DEV)) == expect


# ------------------------------------------------------------------ routing
@pytest.mark.parametrize("T,H,E,k,renorm", [(1000, 512, 8, 2, True), (777, 256, 64, 6, True), (50, 128, 40, 3, False),
                                            (1, 4096, 8, 2, True)])
def test_route_topk(ops, T, H, E, k, renorm):
    x = rand((T, H), seed=1)
    G = rand((E, H), 1 / H ** 0.5, torch.float32, seed=2)
    ids, w, logits = ops.route_topk(x, G, k, renorm)
    lref = oroute.router_logits(f64(x), f64(G))
    assert rel_l2(logits.cpu().numpy(), lref) < 1e-5
    ref_ids, ref_w = oroute.topk_from_logits(logits.cpu().numpy(), k, renorm)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(w.cpu().numpy(), ref_w, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("H,E", [(4096, 8), (2048, 32), (512, 3), (2048, 64)])
def test_route_batch_invariant(ops, dtype, H, E):
    """A token's logits, ids and weights do not depend on the batch around it: the
    fused few-token kernel (T <= 8) and the shared-memory kernel (more tokens) sum
    in the same order; with 64 experts every batch takes the same tiled kernel
    (tensor cores for bf16 tokens)."""
    x = rand((300, H), dtype=dtype, seed=5)
    G = rand((E, H), 1 / H ** 0.5, torch.float32, seed=6)
    k = min(2, E)
    ids_all, w_all, l_all = ops.route_topk(x, G, k, True)
    for T in (1, 3, 8, 9, 40):
        ids, w, logits = ops.route_topk(x[:T].contiguous(), G, k, True)
        assert torch.equal(logits, l_all[:T]), f"T={T}"
        assert torch.equal(ids, ids_all[:T]) and torch.equal(w, w_all[:T]), f"T={T}"


def test_route_matches_reference_make_routing(ops, golden):
    g = golden("routing")
    x = torch.from_numpy(g["hidden"]).to(DEV)
    ids, w, _ = ops.route_topk(x, torch.from_numpy(g["gate_w"]).to(DEV), int(g["k"]), True)
    np.testing.assert_array_equal(ids.cpu().numpy(), g["ids"])
    assert rel_l2(w.cpu().numpy(), g["weights"]) < TOL32


def test_topk_ties_and_equal_logits(ops):
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.5], [2.0, 2.0, 2.0, 2.0], [-1e30, 0.0, -1e30, 5.0]], device=DEV)
    ids, w = ops.topk_from_logits(logits, 2, True)
    ref_ids, ref_w = oroute.topk_from_logits(logits.cpu().numpy(), 2, True)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
    np.testing.assert_allclose(w.cpu().numpy(), ref_w, rtol=1e-6)


# ------------------------------------------------------------------ permutation
# (9000, 2, 8, 0, 32): 18000 pairs in 9 chunks -> the separate placement kernel;
# (1000, 6, 64, 2, 128): 8514 keys -> the sort-based kernels; (1800, 2, ...) and
# (3000, 2, 8, 0, 32): 2 and 3 chunks, placed by the last CTA.
@pytest.mark.parametrize("T,k,E,ns,nT,gbt", [(3000, 2, 8, 1, 5, False), (1000, 6, 64, 2, 128, False),
                                               (700, 1, 4, 0, 3, True), (5, 2, 3, 0, 0, False), (1, 2, 8, 0, 32, False),
                                               (9000, 2, 8, 0, 32, False), (1800, 2, 8, 0, 7, False),
                                               (3000, 2, 8, 0, 32, False)])
def test_permute_bit_exact(ops, T, k, E, ns, nT, gbt):
    rng = np.random.default_rng(T + E)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int64)
    ten = rng.integers(0 if gbt else -1, max(nT, 1), T).astype(np.int32) if (nT or gbt) else None
    w = rng.random((T, k)).astype(np.float32)
    p = ops.permute(torch.from_numpy(ids).to(DEV), torch.from_numpy(w).to(DEV),
                    None if ten is None else torch.from_numpy(ten).to(DEV), n_experts_total=E + ns, n_shared=ns,
                    n_tenants=nT, group_by_tenant=gbt)
    ref = operm.permute(ids, w, ten, E + ns, ns, nT, gbt)
    nt = int(p["num_tiles"].item())
    assert nt == ref["num_tiles"]
    rows = nt * 128
    for name in ("row_token", "row_tenant", "row_pair"):
        np.testing.assert_array_equal(p[name][:rows].cpu().numpy(), ref[name], err_msg=name)
    np.testing.assert_array_equal(p["row_weight"][:rows].cpu().numpy(), ref["row_weight"])
    np.testing.assert_array_equal(p["pair_row"][: T * (k + ns)].cpu().numpy(), ref["pair_row"])
    np.testing.assert_array_equal(p["tile_group"][:nt].cpu().numpy(), ref["tile_group"])
    np.testing.assert_array_equal(p["group_offsets"].cpu().numpy(), ref["group_offsets"])
    np.testing.assert_array_equal(p["group_counts"].cpu().numpy(), ref["group_counts"])
    check_status(ops)


def test_permute_drops_bad_ids_and_reports(ops):
    ids = torch.tensor([[0, 1], [7, 2], [1, -1], [2, 0]], device=DEV)
    ten = torch.tensor([0, 1, 5, -1], dtype=torch.int32, device=DEV)
    p = ops.permute(ids, None, ten, n_experts_total=3, n_tenants=2)
    ref = operm.permute(ids.cpu().numpy(), None, ten.cpu().numpy(), 3, 0, 2)
    assert ref["dropped"] == 3  # expert 7, and both pairs of the token with tenant 5
    np.testing.assert_array_equal(p["pair_row"].cpu().numpy(), ref["pair_row"])
    check_status(ops, 110)


def test_permute_empty(ops):
    p = ops.permute(torch.zeros((0, 2), dtype=torch.int64, device=DEV), None, None, n_experts_total=4)
    assert int(p["num_tiles"].item()) == 0
    np.testing.assert_array_equal(p["group_counts"].cpu().numpy(), np.zeros(4))


# ------------------------------------------------------------------ MoE layer
def _moe_case(T, H, I, E, k, nT, r, ns=0, dtype=torch.bfloat16, seed=0, lora=("w13", "w2"), ten_dist="uniform"):
    rng = np.random.default_rng(seed)
    Et = E + ns
    c = dict(x=rand((T, H), 1.0, dtype, seed), gate_up=rand((Et, 2 * I, H), H ** -0.5, dtype, seed + 1),
             down=rand((Et, H, I), I ** -0.5, dtype, seed + 2), router_w=rand((E, H), H ** -0.5, torch.float32,
                                                                             seed + 3))
    if nT:
        if ten_dist == "zipf":
            p = 1 / (np.arange(nT) + 1) ** 1.1
            ten = rng.choice(nT, T, p=p / p.sum())
        else:
            ten = rng.integers(-1, nT, T)
        c["tenant_ids"] = torch.from_numpy(ten.astype(np.int32)).to(DEV)
        c["lora_scale"] = torch.from_numpy(rng.uniform(0.5, 2.0, nT).astype(np.float32)).to(DEV)
        if "w13" in lora:
            c["lora_a13"] = rand((nT, Et, 2 * r, H), H ** -0.5, dtype, seed + 4)
            c["lora_b13"] = rand((nT, Et, 2 * I, r), r ** -0.5, dtype, seed + 5)
        if "w2" in lora:
            c["lora_a2"] = rand((nT, Et, r, I), I ** -0.5, dtype, seed + 6)
            c["lora_b2"] = rand((nT, Et, H, r), r ** -0.5, dtype, seed + 7)
    return c


def _oracle_moe(c, ids, w, ns=0):
    g = lambda n: None if c.get(n) is None else f64(c[n])
    return omoe.moe_forward(f64(c["x"]), f64(c["gate_up"]), f64(c["down"]), ids, w,
                            tenant_ids=None if c.get("tenant_ids") is None else c["tenant_ids"].cpu().numpy(),
                            n_shared=ns, lora_a13=g("lora_a13"), lora_b13=g("lora_b13"), lora_a2=g("lora_a2"),
                            lora_b2=g("lora_b2"), lora_scale=g("lora_scale"))


@pytest.mark.parametrize("case", [
    dict(T=300, H=256, I=384, E=4, k=2, nT=3, r=16),
    dict(T=257, H=128, I=256, E=3, k=2, nT=7, r=32),
    dict(T=1000, H=256, I=128, E=16, k=4, nT=40, r=16, ns=2, ten_dist="zipf"),
    dict(T=200, H=192, I=320, E=5, k=2, nT=4, r=16, dtype=torch.float16),
    dict(T=64, H=128, I=128, E=4, k=2, nT=3, r=16, lora=("w13",)),
    dict(T=1, H=256, I=256, E=8, k=2, nT=2, r=16),
    dict(T=130, H=136, I=200, E=3, k=3, nT=0, r=0),
    dict(T=600, H=256, I=384, E=6, k=2, nT=9, r=8, ns=1, ten_dist="zipf"),  # rank 8, run-heavy: one-CTA tiles
    dict(T=600, H=1024, I=1024, E=3, k=2, nT=2, r=8, ns=1, ten_dist="zipf"),  # rank 8 on tile pairs
    dict(T=3, H=256, I=256, E=4, k=2, nT=2, r=8),  # rank 8, decode-sized batch
])
def test_moe_forward_vs_oracle(ops, case):
    ns = case.get("ns", 0)
    c = _moe_case(**case)
    y = ops.moe_forward(c["x"], c["gate_up"], c["down"], router_w=c["router_w"], k=case["k"], n_shared=ns,
                        tenant_ids=c.get("tenant_ids"), n_tenants=case["nT"], rank=case["r"],
                        lora_a13=c.get("lora_a13"), lora_b13=c.get("lora_b13"), lora_a2=c.get("lora_a2"),
                        lora_b2=c.get("lora_b2"), lora_scale=c.get("lora_scale"))
    ids, w, _ = ops.route_topk(c["x"], c["router_w"], case["k"], True)
    ref = _oracle_moe(c, ids.cpu().numpy(), w.cpu().numpy(), ns)
    assert rel_l2(f64(y), ref) < TOL16
    check_status(ops)


def test_residual_moe_op_vs_reference_golden(ops, golden):
    g = golden("fallback_moe")
    dt = torch.bfloat16
    hid, gu, dn = (torch.from_numpy(g[n]).to(DEV, dt) for n in ("hidden", "gate_up", "down"))
    tw = torch.from_numpy(g["topk_weights"]).to(DEV)
    tid = torch.from_numpy(g["topk_ids"]).to(DEV)
    y = torch.ops.stageml.residual_moe(hid, gu, dn, tw, tid)
    ref = omoe.fallback_moe(f64(hid), f64(gu), f64(dn), g["topk_weights"], g["topk_ids"])
    assert rel_l2(f64(y), ref) < TOL16
    assert rel_l2(f64(y), g["out"]) < 3e-2  # includes the bf16 rounding of the reference's fp32 inputs


@pytest.mark.parametrize("dtype,wdtype,idt", [(torch.bfloat16, torch.float32, torch.int64),
                                              (torch.float16, torch.float16, torch.int32)])
def test_residual_moe_op(ops, dtype, wdtype, idt):
    T, H, I, E, k = 333, 256, 384, 6, 2
    c = _moe_case(T, H, I, E, k, 0, 0, dtype=dtype, seed=5)
    rng = np.random.default_rng(5)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    w = rng.random((T, k)).astype(np.float32)
    y = ops.residual_moe(c["x"], c["gate_up"], c["down"], torch.from_numpy(w).to(DEV, wdtype),
                         torch.from_numpy(ids).to(DEV, idt))
    w_used = torch.from_numpy(w).to(wdtype).float().numpy()
    ref = omoe.fallback_moe(f64(c["x"]), f64(c["gate_up"]), f64(c["down"]), w_used, ids)
    assert rel_l2(f64(y), ref) < TOL16


def test_moe_forward_is_deterministic_and_permutation_invariant(ops):
    c = _moe_case(T=500, H=256, I=256, E=8, k=2, nT=6, r=16, seed=9)
    kw = dict(router_w=c["router_w"], k=2, tenant_ids=c["tenant_ids"], n_tenants=6, rank=16,
              lora_a13=c["lora_a13"], lora_b13=c["lora_b13"], lora_a2=c["lora_a2"], lora_b2=c["lora_b2"],
              lora_scale=c["lora_scale"])
    y1 = ops.moe_forward(c["x"], c["gate_up"], c["down"], **kw)
    y2 = ops.moe_forward(c["x"], c["gate_up"], c["down"], **kw)
    assert torch.equal(y1, y2)
    perm = torch.randperm(500, generator=torch.Generator().manual_seed(0)).to(DEV)
    kw["tenant_ids"] = c["tenant_ids"][perm].contiguous()
    y3 = ops.moe_forward(c["x"][perm].contiguous(), c["gate_up"], c["down"], **kw)
    assert torch.equal(y3, y1[perm])


def test_moe_forward_zero_lora_scale_equals_no_lora(ops):
    c = _moe_case(T=200, H=128, I=256, E=4, k=2, nT=3, r=16, seed=11)
    y0 = ops.moe_forward(c["x"], c["gate_up"], c["down"], router_w=c["router_w"], k=2)
    y1 = ops.moe_forward(c["x"], c["gate_up"], c["down"], router_w=c["router_w"], k=2, tenant_ids=c["tenant_ids"],
                         n_tenants=3, rank=16, lora_a13=c["lora_a13"], lora_b13=c["lora_b13"], lora_a2=c["lora_a2"],
                         lora_b2=c["lora_b2"], lora_scale=torch.zeros(3, device=DEV))
    assert torch.equal(y0, y1)


def test_decode_calls_back_to_back_match_synchronized_calls(ops):
    """Decode-sized calls (at most 16 routed rows) run their kernel chain as
    programmatic dependent launches; issued back to back on one stream, with LoRA on
    w1/w3/w2, on w1/w3 only and off, they give the same bits as the same calls with a
    device synchronization after each."""
    full = _moe_case(T=48, H=256, I=256, E=8, k=2, nT=3, r=16, seed=13)
    w13 = _moe_case(T=48, H=256, I=256, E=8, k=2, nT=3, r=16, seed=13, lora=("w13",))

    def call(i):
        c = (full, w13, full)[i % 3]
        x = c["x"][2 * i:2 * i + 2]
        kw = dict(router_w=c["router_w"], k=2)
        if i % 3 != 2:
            kw.update(tenant_ids=c["tenant_ids"][2 * i:2 * i + 2], n_tenants=3, rank=16, lora_a13=c["lora_a13"],
                      lora_b13=c["lora_b13"], lora_a2=c.get("lora_a2"), lora_b2=c.get("lora_b2"),
                      lora_scale=c["lora_scale"])
        return ops.moe_forward(x, c["gate_up"], c["down"], **kw)

    ref = []
    for i in range(24):
        ref.append(call(i))
        torch.cuda.synchronize()
    out = [call(i) for i in range(24)]
    torch.cuda.synchronize()
    for i in range(24):
        assert torch.equal(out[i], ref[i]), f"call {i}"
    check_status(ops)


def test_large_calls_back_to_back_match_synchronized_calls(ops):
    """Larger batches run their chains (permutation, plans, shrinks, grouped GEMMs,
    combine) as programmatic dependent launches too. Issued back to back on one stream,
    interleaving MoE layers (CTA pairs with half units and odd tiles beside them, LoRA on
    all projections and off) with mixed-adapter linear layers (direct and grouped rows),
    the calls give the same bits as with a device synchronization after each."""
    moe = _moe_case(T=700, H=512, I=512, E=4, k=2, nT=3, r=16, seed=21)
    rng = np.random.default_rng(22)
    x = rand((384, 512), 1.0, torch.bfloat16, 23)
    Wb = rand((3, 768, 512), 512 ** -0.5, torch.bfloat16, 24)
    A = rand((4, 16, 512), 512 ** -0.5, torch.bfloat16, 25)
    B = rand((4, 768, 16), 16 ** -0.5, torch.bfloat16, 26)
    sc = torch.from_numpy(rng.uniform(0.5, 2, 4).astype(np.float32)).to(DEV)
    ten = torch.from_numpy(rng.integers(-1, 4, 384).astype(np.int32)).to(DEV)
    grp = torch.from_numpy(rng.integers(0, 3, 384).astype(np.int32)).to(DEV)

    def call(i):
        kind = i % 4
        if kind == 0:
            return ops.moe_forward(moe["x"], moe["gate_up"], moe["down"], router_w=moe["router_w"], k=2,
                                   tenant_ids=moe["tenant_ids"], n_tenants=3, rank=16, lora_a13=moe["lora_a13"],
                                   lora_b13=moe["lora_b13"], lora_a2=moe["lora_a2"], lora_b2=moe["lora_b2"],
                                   lora_scale=moe["lora_scale"])
        if kind == 1:
            return ops.lora_linear(x, Wb[:1], row_tenant=ten, n_tenants=4, rank=16, lora_a=A, lora_b=B, lora_scale=sc)
        if kind == 2:
            return ops.moe_forward(moe["x"][: 600 - 37 * (i % 3)], moe["gate_up"], moe["down"],
                                   router_w=moe["router_w"], k=2)
        return ops.lora_linear(x, Wb, row_group=grp, row_tenant=ten, n_tenants=4, rank=16, lora_a=A, lora_b=B,
                               lora_scale=sc)

    ref = []
    for i in range(16):
        ref.append(call(i))
        torch.cuda.synchronize()
    out = [call(i) for i in range(16)]
    torch.cuda.synchronize()
    for i in range(16):
        assert torch.equal(out[i], ref[i]), f"call {i}"
    check_status(ops)


def test_decode_rows_do_not_depend_on_the_batch(ops):
    """A token's output from a decode-sized call has the same bits alone as inside a
    batch of 8: the skinny GEMMs' per-row sums do not depend on the batch (the
    batch also takes the kernel variant for more than 8 rows per tile)."""
    c = _moe_case(T=8, H=512, I=14336, E=2, k=2, nT=2, r=16, seed=17)
    kw = dict(router_w=c["router_w"], k=2, n_tenants=2, rank=16, lora_a13=c["lora_a13"], lora_b13=c["lora_b13"],
              lora_a2=c["lora_a2"], lora_b2=c["lora_b2"], lora_scale=c["lora_scale"])
    y = ops.moe_forward(c["x"], c["gate_up"], c["down"], tenant_ids=c["tenant_ids"], **kw)
    for t in range(8):
        yt = ops.moe_forward(c["x"][t:t + 1], c["gate_up"], c["down"], tenant_ids=c["tenant_ids"][t:t + 1], **kw)
        assert torch.equal(yt[0], y[t]), f"token {t}"
    ids, w, _ = ops.route_topk(c["x"], c["router_w"], 2, True)
    assert rel_l2(f64(y), _oracle_moe(c, ids.cpu().numpy(), w.cpu().numpy())) < TOL16
    check_status(ops)


def test_moe_forward_empty_batch(ops):
    c = _moe_case(T=1, H=128, I=128, E=4, k=2, nT=0, r=0)
    y = ops.moe_forward(c["x"][:0], c["gate_up"], c["down"], router_w=c["router_w"], k=2)
    assert y.shape == (0, 128)


# ------------------------------------------------------------------ MoE single linear
def test_moe_linear_dynamic_and_materialized(ops):
    T, K, N, E, k, nT, r = 190, 64, 48, 4, 2, 3, 16
    rng = np.random.default_rng(7)
    x = rand((T, K), seed=21)
    W = rand((E, N, K), K ** -0.5, seed=22)
    bias = rand((E, N), 0.1, seed=23)
    A = rand((nT, E, r, K), K ** -0.5, seed=24)
    B = rand((nT, E, N, r), r ** -0.5, seed=25)
    sc = torch.tensor([0.5, 1.0, 2.0], device=DEV)
    ids = torch.from_numpy(np.stack([rng.permutation(E)[:k] for _ in range(T)])).to(DEV)
    w = torch.from_numpy(rng.random((T, k)).astype(np.float32)).to(DEV)
    ten = torch.from_numpy(rng.integers(0, nT, T).astype(np.int32)).to(DEV)
    y = ops.moe_linear(x, W, ids, w, bias=bias, tenant_ids=ten, n_experts=E, n_tenants=nT, rank=r, lora_a=A, lora_b=B,
                       lora_scale=sc)
    ref = omoe.moe_linear(f64(x), f64(W), ids.cpu().numpy(), w.cpu().numpy(), bias=f64(bias),
                          tenant_ids=ten.cpu().numpy(), lora_a=f64(A), lora_b=f64(B), lora_scale=sc.cpu().numpy())
    assert rel_l2(f64(y), ref) < TOL16
    merged = torch.stack([ops.lora_fold(W, A[a], B[a], torch.full((E,), float(sc[a]), device=DEV)) for a in range(nT)])
    y2 = ops.moe_linear(x, merged.view(nT * E, N, K), ids, w, bias=bias, tenant_ids=ten, n_experts=E,
                        group_by_tenant=True, n_tenants=nT)
    ref2 = omoe.moe_linear(f64(x), None, ids.cpu().numpy(), w.cpu().numpy(), bias=f64(bias),
                           tenant_ids=ten.cpu().numpy(), merged=f64(merged))
    assert rel_l2(f64(y2), ref2) < TOL16
    assert rel_l2(f64(y2), ref) < 2e-2


# ------------------------------------------------------------------ dense LoRA linear
@pytest.mark.parametrize("M,K,N,nT,r,G,dtype", [(333, 256, 512, 5, 16, 1, torch.bfloat16),
                                                (500, 256, 384, 40, 16, 1, torch.float16),
                                                (300, 128, 256, 9, 32, 1, torch.bfloat16),
                                                (400, 256, 256, 4, 16, 3, torch.bfloat16),
                                                (256, 512, 512, 64, 16, 9, torch.bfloat16),
                                                (333, 256, 384, 6, 8, 1, torch.bfloat16),
                                                (400, 256, 256, 5, 8, 3, torch.float16),
                                                (7, 72, 24, 0, 0, 1, torch.bfloat16)])
def test_lora_linear(ops, M, K, N, nT, r, G, dtype):
    rng = np.random.default_rng(M + N)
    x = rand((M, K), 1.0, dtype, 31)
    Wb = rand((G, N, K), K ** -0.5, dtype, 32)
    bias = rand((N,), 0.1, dtype, 33)
    grp = rng.integers(0, G, M).astype(np.int32)
    kw = dict(bias=bias)
    ref = np.einsum("mk,mnk->mn", f64(x), f64(Wb)[grp]) + f64(bias)
    if G > 1:
        kw["row_group"] = torch.from_numpy(grp).to(DEV)
    if nT:
        ten = np.where(grp == 0, rng.integers(-1, nT, M), -1).astype(np.int32)
        A = rand((nT, r, K), K ** -0.5, dtype, 34)
        B = rand((nT, N, r), r ** -0.5, dtype, 35)
        sc = torch.from_numpy(rng.uniform(0.5, 2, nT).astype(np.float32)).to(DEV)
        kw.update(row_tenant=torch.from_numpy(ten).to(DEV), n_tenants=nT, rank=r, lora_a=A, lora_b=B, lora_scale=sc)
        m = ten >= 0
        s = np.einsum("mk,mrk->mr", f64(x)[m], f64(A)[ten[m]]) * sc.cpu().numpy()[ten[m]][:, None]
        ref[m] += np.einsum("mr,mnr->mn", s, f64(B)[ten[m]])
    y = ops.lora_linear(x, Wb, **kw)
    assert rel_l2(f64(y), ref) < TOL16
    check_status(ops)


def test_lora_linear_bad_tenant_is_reported(ops):
    x = rand((64, 64), seed=41)
    W = rand((1, 64, 64), 0.1, seed=42)
    A = rand((2, 16, 64), 0.1, seed=43)
    B = rand((2, 64, 16), 0.1, seed=44)
    ten = torch.tensor([0, 1, 5] + [0] * 61, dtype=torch.int32, device=DEV)
    y = ops.lora_linear(x, W, row_tenant=ten, n_tenants=2, rank=16, lora_a=A, lora_b=B,
                        lora_scale=torch.ones(2, device=DEV))
    check_status(ops, 110)
    ref = f64(x) @ f64(W)[0].T  # row 2 (tenant 5) gets no LoRA
    assert rel_l2(f64(y)[2], ref[2]) < TOL16


# ------------------------------------------------------------------ fold
@pytest.mark.parametrize("dtype,layout,rows,cols,r,batch,bcast", [
    (torch.bfloat16, 0, 512, 384, 16, 3, True), (torch.float16, 0, 300, 200, 8, 2, False),
    (torch.bfloat16, 1, 256, 512, 16, 1, True), (torch.float32, 0, 100, 60, 4, 2, True),
    (torch.float32, 1, 1024, 512, 16, 1, True), (torch.bfloat16, 0, 12, 20, 3, 1, True),
    (torch.float32, 0, 70, 36, 24, 2, False), (torch.float32, 1, 33, 13, 8, 1, True),
    (torch.bfloat16, 0, 130, 264, 40, 4, True), (torch.float16, 1, 200, 136, 16, 3, False)])
def test_lora_fold(ops, dtype, layout, rows, cols, r, batch, bcast):
    W = rand((rows, cols) if bcast else (batch, rows, cols), 1.0, dtype, 51)
    if layout == 0:
        A = rand((batch, r, cols), 1.0, dtype, 52)
        B = rand((batch, rows, r), 1.0, dtype, 53)
    else:
        A = rand((batch, rows, r), 1.0, dtype, 52)
        B = rand((batch, r, cols), 1.0, dtype, 53)
    sc = torch.linspace(0.5, 2.0, batch, device=DEV)
    out = ops.lora_fold(W, A, B, sc, layout)
    for b in range(batch):
        Wb = f64(W) if bcast else f64(W)[b]
        ref = olora.lora_fold(Wb, f64(A)[b], f64(B)[b], float(sc[b]), layout)
        tol = TOL32 if dtype == torch.float32 else 4e-3
        assert rel_l2(f64(out)[b], ref) < tol


def test_fold_known_answer(ops, golden):
    g = golden("fold")
    for dt in (torch.float32, torch.bfloat16):
        out = ops.lora_fold(torch.from_numpy(g["known_W"]).to(DEV, dt), torch.from_numpy(g["known_A"]).to(DEV, dt),
                            torch.from_numpy(g["known_B"]).to(DEV, dt), float(g["known_scale"]), 0)
        np.testing.assert_array_equal(out.float().cpu().numpy(), g["known_out"])
    out = ops.lora_fold(torch.from_numpy(g["W"]).to(DEV), torch.from_numpy(g["A"]).to(DEV),
                        torch.from_numpy(g["B"]).to(DEV), float(g["scale"]), 0)
    assert rel_l2(out.cpu().numpy(), g["out"]) < TOL32


# ------------------------------------------------------------------ config 1 (fp32)
def test_single_lora_gemv_config1(ops):
    from stageml_b200.workloads import make_single_lora

    w = make_single_lora(seed=0, device=DEV, gen_device="cpu")
    y = ops.lora_gemv_f32(w["x"], w["W"], w["A"], w["B"], w["scale"])
    ref = olora.single_lora(f64(w["x"]), f64(w["W"]), f64(w["A"]), f64(w["B"]), w["scale"])
    assert rel_l2(f64(y), ref) < TOL32
    Wf = ops.lora_fold(w["W"], w["A"], w["B"], w["scale"], 1)
    yf = ops.lora_gemv_f32(w["x"], Wf)
    assert rel_l2(f64(yf), ref) < TOL32
    assert rel_l2(f64(yf), f64(y)) < TOL32


@pytest.mark.parametrize("M,din,dout,r", [(1, 4096, 4096, 16), (3, 1000, 770, 8), (4, 64, 4099, 4),
                                         (7, 3001, 512, 16), (16, 4096, 1030, 32), (1, 5, 3, 1)])
def test_single_lora_gemv_shapes(ops, M, din, dout, r):
    """The three row templates of the split-K GEMV (1, <= 4, <= 16 rows of x), outputs that are
    not a multiple of 4 (scalar tail), slices that do not divide the input, fp32 within 1e-5."""
    g = torch.Generator().manual_seed(M * 7 + din)
    x = torch.randn(M, din, generator=g).to(DEV)
    W = (torch.randn(din, dout, generator=g) / din ** 0.5).to(DEV)
    A = (torch.randn(din, r, generator=g) / din ** 0.5).to(DEV)
    B = (torch.randn(r, dout, generator=g) / r ** 0.5).to(DEV)
    y = ops.lora_gemv_f32(x, W, A, B, 1.5)
    ref = olora.single_lora(f64(x), f64(W), f64(A), f64(B), 1.5)
    assert rel_l2(f64(y), ref) < TOL32
    y0 = ops.lora_gemv_f32(x, W)
    assert rel_l2(f64(y0), f64(x) @ f64(W)) < TOL32
    assert torch.equal(ops.lora_gemv_f32(x, W, A, B, 1.5), y)  # deterministic


def test_single_lora_vs_reference_golden(ops, golden):
    g = golden("single_lora")
    t = lambda n: torch.from_numpy(g[n]).to(DEV)
    y = ops.lora_gemv_f32(t("x"), t("W"), t("A"), t("B"), float(g["scale"]))
    assert rel_l2(y.cpu().numpy(), g["y"]) < TOL32
    yf = ops.lora_gemv_f32(t("x"), ops.lora_fold(t("W"), t("A"), t("B"), float(g["scale"]), 1))
    assert rel_l2(yf.cpu().numpy(), g["y_residual"]) < TOL32


# ------------------------------------------------------------------ FP8 weights
def test_quantize_e4m3_rows_bit_exact(ops):
    w = rand((300, 1000), 0.05, torch.bfloat16, 61)
    w[7] = 0
    q, s = ops.quantize_e4m3_rows(w)
    rq, rs = numerics.quantize_e4m3_rows(w.float().cpu().numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), rq)


def _fp8_weights(c, ops):
    """e4m3 codes + per-row scales of the case's weights, and the 16-bit weights they dequantise to."""
    out = {}
    for n in ("gate_up", "down"):
        w = c[n]
        q, s = ops.quantize_e4m3_rows(w.reshape(-1, w.shape[-1]))
        out[n] = q.view(w.shape)
        out[n + "_scale"] = s.view(w.shape[:-1]).contiguous()
        out[n + "_deq"] = (q.float() * s[:, None]).to(w.dtype).view(w.shape)
    return out


@pytest.mark.parametrize("case", [
    dict(T=300, H=256, I=384, E=4, k=2, nT=3, r=16),
    dict(T=200, H=144, I=208, E=5, k=2, nT=4, r=32, dtype=torch.float16),
    dict(T=1000, H=256, I=128, E=16, k=4, nT=40, r=16, ns=2, ten_dist="zipf"),
    dict(T=130, H=128, I=176, E=3, k=3, nT=0, r=0),
    dict(T=1, H=256, I=256, E=8, k=2, nT=2, r=16),
    dict(T=700, H=256, I=192, E=8, k=3, nT=20, r=8, ns=1, ten_dist="zipf"),
])
def test_moe_forward_fp8_weights(ops, case):
    """e4m3 weights, fp32 per-output-channel scales (weight-only FP8: dequantised before the MMA).

    Checked against the oracle on the dequantised weights (rel-L2 <= 1e-2) and bit-exactly
    against the 16-bit path given the same weights dequantised on the host.
    """
    ns = case.get("ns", 0)
    c = _moe_case(**case)
    f = _fp8_weights(c, ops)
    kw = dict(router_w=c["router_w"], k=case["k"], n_shared=ns, tenant_ids=c.get("tenant_ids"), n_tenants=case["nT"],
              rank=case["r"], lora_a13=c.get("lora_a13"), lora_b13=c.get("lora_b13"), lora_a2=c.get("lora_a2"),
              lora_b2=c.get("lora_b2"), lora_scale=c.get("lora_scale"))
    y8 = ops.moe_forward(c["x"], f["gate_up"], f["down"], gate_up_scale=f["gate_up_scale"],
                         down_scale=f["down_scale"], **kw)
    y16 = ops.moe_forward(c["x"], f["gate_up_deq"], f["down_deq"], **kw)
    check_status(ops)
    assert torch.equal(y8, y16)
    ids, w, _ = ops.route_topk(c["x"], c["router_w"], case["k"], True)
    gq = numerics.dequantize_e4m3_rows(f["gate_up"].view(torch.uint8).reshape(-1, case["H"]).cpu().numpy(),
                                       f["gate_up_scale"].reshape(-1).cpu().numpy())
    dq = numerics.dequantize_e4m3_rows(f["down"].view(torch.uint8).reshape(-1, case["I"]).cpu().numpy(),
                                       f["down_scale"].reshape(-1).cpu().numpy())
    c8 = dict(c, gate_up=torch.from_numpy(gq.reshape(tuple(c["gate_up"].shape))),
              down=torch.from_numpy(dq.reshape(tuple(c["down"].shape))))
    ref = _oracle_moe(c8, ids.cpu().numpy(), w.cpu().numpy(), ns)
    assert rel_l2(f64(y8), ref) < TOL16


def test_moe_forward_fp8_needs_scales(ops):
    c = _moe_case(T=16, H=128, I=128, E=2, k=1, nT=0, r=0)
    f = _fp8_weights(c, ops)
    with pytest.raises(RuntimeError, match="scale"):
        ops.moe_forward(c["x"], f["gate_up"], f["down"], router_w=c["router_w"], k=1)
