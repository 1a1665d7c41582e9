"""Properties of the token -> expert permutation plan (no GPU needed).

The oracle's plan (oracle/permute.py) is the checker for the CUDA permutation,
bit for bit, in the GPU tests; it is pinned to the reference's grouping by the
golden vectors. Here it is checked against the definition itself on random
shapes, including out-of-range expert and tenant ids, and the workspace bound
that sizes the plan buffers is checked against the library's own
stageml_plan_rows_cap.
"""

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from oracle import permute as operm
from stageml_b200._native import load_capi


@st.composite
def routing(draw):
    T = draw(st.integers(0, 300))
    E = draw(st.integers(1, 12))
    k = draw(st.integers(1, min(E, 4)))
    n_shared = draw(st.integers(0, 2))
    n_tenants = draw(st.integers(0, 9))
    seed = draw(st.integers(0, 2**31 - 1))
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]) if T else np.zeros((0, k), np.int64)
    if T and draw(st.booleans()):  # a few out-of-range expert ids
        bad = rng.random(ids.shape) < 0.05
        ids = np.where(bad, rng.choice([-1, E, E + 3], size=ids.shape), ids)
    w = rng.random((T, k)).astype(np.float32)
    ten = rng.integers(-1, n_tenants, size=T) if n_tenants else np.full(T, -1)
    if T and n_tenants and draw(st.booleans()):  # a few out-of-range tenant ids
        ten = np.where(rng.random(T) < 0.05, n_tenants + 1, ten)
    return ids.astype(np.int64), w, ten.astype(np.int64), E, k, n_shared, n_tenants


@settings(max_examples=80, deadline=None)
@given(routing())
def test_plan_matches_its_definition(case):
    ids, w, ten, E, k, n_shared, n_tenants = case
    T = ids.shape[0]
    kk = k + n_shared
    E_tot = E + n_shared
    p = operm.permute(ids, w, ten, E_tot, n_shared, n_tenants)
    P = T * kk

    # which pairs are kept, by the stated rule
    expert = np.empty(P, np.int64)
    weight = np.ones(P, np.float32)
    tenant = np.repeat(ten, kk)
    for t in range(T):
        for j in range(kk):
            expert[t * kk + j] = ids[t, j] if j < k else E + j - k
            if j < k:
                weight[t * kk + j] = w[t, j]
    routed = (np.arange(P) % kk) < k
    bad = (routed & ((expert < 0) | (expert >= E))) | (tenant >= n_tenants) | (tenant < -1)
    assert p["dropped"] == int(bad.sum())
    assert np.all(p["pair_row"][bad] == -1)

    # every kept pair sits in exactly one row, and pair_row inverts row_pair
    rp = p["row_pair"]
    filled = rp >= 0
    assert sorted(rp[filled].tolist()) == np.flatnonzero(~bad).tolist()
    assert np.all(p["pair_row"][rp[filled]] == np.flatnonzero(filled))
    assert np.all(p["row_token"][filled] == rp[filled] // kk)
    assert np.array_equal(p["row_weight"][filled], weight[rp[filled]])
    assert np.all(p["row_token"][~filled] == -1) and np.all(p["row_weight"][~filled] == 0)

    # 128-row padded segments in expert order, stable by (tenant, pair index) inside
    off = p["group_offsets"]
    assert off[0] == 0 and np.all(off % 128 == 0) and len(off) == E_tot + 1
    for g in range(E_tot):
        seg = rp[off[g]:off[g + 1]]
        n = int(p["group_counts"][g])
        assert (off[g + 1] - off[g]) == (n + 127) // 128 * 128
        assert np.all(seg[:n] >= 0) and np.all(seg[n:] == -1)
        assert np.all(expert[seg[:n]] == g)
        keys = list(zip(tenant[seg[:n]].tolist(), seg[:n].tolist()))
        assert keys == sorted(keys)
        assert np.all(p["tile_group"][off[g] // 128:off[g + 1] // 128] == g)
    assert p["num_tiles"] * 128 == off[-1]

    # the plan fits the buffers sized by the bound
    assert off[-1] <= operm.rows_cap(P, E_tot)


@pytest.mark.parametrize("groups", [1, 2, 3, 8, 64, 66, 1000])
def test_rows_cap_matches_the_library(groups):
    lib = load_capi()
    for P in [0, 1, 2, 3, 127, 128, 129, 4095, 4096, 4097, 65536, 1 << 20]:
        assert lib.stageml_plan_rows_cap(P, groups) == operm.rows_cap(P, groups), (P, groups)
