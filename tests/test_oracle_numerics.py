"""Number formats and routing rules of the oracle, checked on the CPU."""

import numpy as np
import torch

from oracle import numerics, route


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(10000) * 10.0 ** rng.integers(-20, 20, 10000),
                        np.array([0.0, -0.0, 1.0, 65504.0, 1e-40, 3.0e38], dtype=np.float32)]).astype(np.float32)
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(numerics.round_bf16(x), ref)


def test_e4m3_encode_matches_torch_in_range():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.uniform(-448, 448, 20000), rng.standard_normal(20000) * 0.01,
                        np.array([0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 1.0625, 1.1875])]).astype(np.float32)
    codes = numerics.encode_e4m3(x)
    ref = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(codes, ref)
    np.testing.assert_array_equal(numerics.decode_e4m3(codes),
                                  torch.from_numpy(ref).view(torch.float8_e4m3fn).float().numpy())


def test_e4m3_saturates():
    codes = numerics.encode_e4m3(np.array([1000.0, -1e9, 449.0, 464.0, np.inf], dtype=np.float32))
    np.testing.assert_array_equal(numerics.decode_e4m3(codes), [448.0, -448.0, 448.0, 448.0, 448.0])


def test_quantize_rows_scale_and_reconstruction():
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((16, 64)) / 8).astype(np.float32)
    w[3] = 0.0
    q, s = numerics.quantize_e4m3_rows(w)
    assert s[3] == 1.0
    np.testing.assert_allclose(s[0], np.abs(w[0]).max() / 448.0, rtol=1e-7)
    deq = numerics.dequantize_e4m3_rows(q, s)
    assert np.abs(deq - w).max() <= np.abs(w).max() * 2 ** -4 + 1e-12
    assert np.abs(numerics.decode_e4m3(q)).max() <= 448.0


def test_topk_ties_go_to_lower_expert():
    logits = np.array([[1.0, 3.0, 3.0, 0.5], [2.0, 2.0, 2.0, 2.0]], dtype=np.float32)
    ids, w = route.topk_from_logits(logits, 2)
    np.testing.assert_array_equal(ids, [[1, 2], [0, 1]])
    np.testing.assert_allclose(w, [[0.5, 0.5], [0.5, 0.5]], rtol=1e-6)


def test_renormalize_matches_reference_rule():
    w = np.array([[0.2, 0.3], [0.0, 0.0]], dtype=np.float32)
    np.testing.assert_allclose(route.normalize_routing_weights(w), [[0.4, 0.6], [0.0, 0.0]])


def test_moe_forward_zero_lora_equals_fallback():
    from oracle import moe

    rng = np.random.default_rng(3)
    T, H, I, E, k, nT, r = 10, 16, 8, 3, 2, 2, 4
    x = rng.standard_normal((T, H))
    gu = rng.standard_normal((E, 2 * I, H)) * 0.2
    dn = rng.standard_normal((E, H, I)) * 0.2
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    w = rng.random((T, k))
    zeros = dict(lora_a13=np.zeros((nT, E, 2 * r, H)), lora_b13=rng.standard_normal((nT, E, 2 * I, r)),
                 lora_a2=np.zeros((nT, E, r, I)), lora_b2=rng.standard_normal((nT, E, H, r)),
                 lora_scale=np.ones(nT))
    y = moe.moe_forward(x, gu, dn, ids, w, tenant_ids=rng.integers(0, nT, T), **zeros)
    np.testing.assert_allclose(y, moe.fallback_moe(x, gu, dn, w, ids), rtol=1e-12, atol=1e-12)


def test_shared_experts_are_always_on_with_weight_one():
    from oracle import moe

    rng = np.random.default_rng(4)
    T, H, I, E, k = 6, 8, 8, 3, 1
    x = rng.standard_normal((T, H))
    gu = rng.standard_normal((E + 1, 2 * I, H))
    dn = rng.standard_normal((E + 1, H, I))
    ids = rng.integers(0, E, (T, k))
    w = np.ones((T, k))
    y = moe.moe_forward(x, gu, dn, ids, w, n_shared=1)
    ids2 = np.concatenate([ids, np.full((T, 1), E)], 1)
    y2 = moe.moe_forward(x, gu, dn, ids2, np.ones((T, 2)))
    np.testing.assert_allclose(y, y2, rtol=1e-12)


def test_oracle_fold_slots_equal_dynamic_lora():
    """A (tenant, expert) pair on a folded weight set (W + s B A on w1, w3 and w2) gives the
    layer output of the same pair with dynamic LoRA, the semantics the golden vectors pin;
    the permutation puts folded pairs in their own groups with no LoRA tenant."""
    from oracle import moe as omoe
    from oracle import permute as operm

    rng = np.random.default_rng(5)
    T, H, I, E, k, nT, r, ns = 40, 16, 24, 3, 2, 4, 4, 1
    Et = E + ns
    x = rng.normal(size=(T, H))
    gu = rng.normal(size=(Et, 2 * I, H)) / 4
    dn = rng.normal(size=(Et, H, I)) / 5
    a13 = rng.normal(size=(nT, Et, 2 * r, H)) / 4
    b13 = rng.normal(size=(nT, Et, 2 * I, r)) / 2
    a2 = rng.normal(size=(nT, Et, r, I)) / 5
    b2 = rng.normal(size=(nT, Et, H, r)) / 2
    sc = np.array([0.5, 1.0, 1.5, 2.0])
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    w = rng.random((T, k))
    ten = rng.integers(-1, nT, T)
    fold = np.full((nT, Et), -1)
    folds = [(1, 0), (1, 2), (3, 3), (2, 1)]  # (tenant, expert), a shared expert among them
    gu_f, dn_f = [], []
    for s, (a, e) in enumerate(folds):
        fold[a, e] = s
        g = gu[e].copy()
        g[:I] += sc[a] * b13[a, e, :I] @ a13[a, e, :r]
        g[I:] += sc[a] * b13[a, e, I:] @ a13[a, e, r:]
        gu_f.append(g)
        dn_f.append(dn[e] + sc[a] * b2[a, e] @ a2[a, e])
    lora = dict(lora_a13=a13, lora_b13=b13, lora_a2=a2, lora_b2=b2, lora_scale=sc)
    ref = omoe.moe_forward(x, gu, dn, ids, w, tenant_ids=ten, n_shared=ns, **lora)
    got = omoe.moe_forward(x, np.concatenate([gu, np.stack(gu_f)]), np.concatenate([dn, np.stack(dn_f)]), ids, w,
                           tenant_ids=ten, n_shared=ns, fold_slot=fold, **lora)
    np.testing.assert_allclose(got, ref, rtol=1e-10, atol=1e-10)
    plan = operm.permute(ids, w, ten, Et, ns, nT, fold_slot=fold, n_fold=len(folds))
    assert len(plan["group_counts"]) == Et + len(folds)
    for s, (a, e) in enumerate(folds):
        rows = np.arange(plan["group_offsets"][Et + s], plan["group_offsets"][Et + s] + plan["group_counts"][Et + s])
        toks = plan["row_token"][rows]
        assert np.all(ten[toks] == a) and np.all(plan["row_tenant"][rows] == -1)
        n_expected = int(np.sum(ten == a)) if e >= E else int(np.sum((ten == a)[:, None] & (ids == e)))
        assert rows.size == n_expected
    bad = fold.copy()
    bad[0, 0] = len(folds)  # out of range: the pair is dropped
    assert operm.permute(ids, w, ten, Et, ns, nT, fold_slot=bad, n_fold=len(folds))["dropped"] == int(
        np.sum((ten == 0)[:, None] & (ids == 0)))
