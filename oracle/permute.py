"""Token -> expert permutation restated in numpy (test infrastructure).

The reference groups the (token, slot) pairs of each expert with one
torch.nonzero per (slot, expert) (benchmarks/multitenant_bta_system_bench.py:401-406);
it builds no explicit permutation. The permutation of this path is defined as:
pairs p = t*(k+n_shared) + j (slot j < k: expert ids[t, j], weight w[t, j];
slot j >= k: shared expert E + j - k, weight 1) sorted stably by the key
(expert, tenant + 1) -- or (tenant*E_tot + expert) with group_by_tenant --
with each group's rows padded to a multiple of 128. Pairs whose expert or
tenant id is out of range are dropped (pair_row = -1). With a fold map
fold_slot [n_tenants, E_tot], a pair whose (tenant, expert) entry is s >= 0
belongs to weight group E_tot + s (after every expert group), sorts by that
group alone and carries no LoRA tenant; an entry outside [-1, n_fold) drops it.
"""

from __future__ import annotations

import numpy as np


def rows_cap(num_pairs: int, n_groups: int) -> int:
    if num_pairs <= 0:
        return 128
    g = min(n_groups, num_pairs)
    return (num_pairs + g * 127 + 127) // 128 * 128


def permute(ids, weights, tenant_ids, n_experts_total: int, n_shared: int = 0, n_tenants: int = 0,
            group_by_tenant: bool = False, fold_slot=None, n_fold: int = 0) -> dict:
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    kk = k + n_shared
    P = T * kk
    E_routed = n_experts_total - n_shared
    t_of = np.repeat(np.arange(T), kk)
    j_of = np.tile(np.arange(kk), T)
    expert = np.empty(P, dtype=np.int64)
    wt = np.ones(P, dtype=np.float32)
    routed = j_of < k
    expert[routed] = ids.reshape(-1)[(t_of * k + j_of)[routed]]
    expert[~routed] = E_routed + (j_of[~routed] - k)
    if weights is not None:
        wt[routed] = np.asarray(weights, dtype=np.float32).reshape(-1)[(t_of * k + j_of)[routed]]
    ten = np.full(T, -1, dtype=np.int64) if tenant_ids is None else np.asarray(tenant_ids, dtype=np.int64)
    tenant = ten[t_of]
    bad = (routed & ((expert < 0) | (expert >= E_routed))) | (tenant < -1) | (tenant >= n_tenants)
    if group_by_tenant:
        bad |= tenant < 0
        n_groups = n_tenants * n_experts_total
        group = np.where(bad, 0, tenant * n_experts_total + expert)
        key = group
    else:
        n_groups = n_experts_total
        group = np.where(bad, 0, expert)
        key = group * (n_tenants + 1) + (tenant + 1)
    lora_tenant = np.full(P, -1, dtype=np.int64) if group_by_tenant else tenant.copy()
    if fold_slot is not None:
        fs = np.asarray(fold_slot, dtype=np.int64)
        ok = ~bad & (tenant >= 0)
        slot = np.full(P, -1, dtype=np.int64)
        slot[ok] = fs[tenant[ok], expert[ok]]
        bad |= (slot < -1) | (slot >= n_fold)
        fold = ~bad & (slot >= 0)
        group = np.where(fold, n_groups + slot, group)
        key = np.where(fold, n_groups * (n_tenants + 1) + slot, key)
        lora_tenant = np.where(fold, -1, lora_tenant)
        n_groups += n_fold
    key = np.where(bad, np.iinfo(np.int64).max, key)
    order = np.lexsort((np.arange(P), key))
    order = order[~bad[order]]
    counts = np.bincount(group[order], minlength=n_groups)[:n_groups]
    padded = (counts + 127) // 128 * 128
    offsets = np.concatenate([[0], np.cumsum(padded)]).astype(np.int64)
    num_tiles = int(offsets[-1] // 128)
    nrows = num_tiles * 128
    row_token = np.full(nrows, -1, dtype=np.int64)
    row_tenant = np.full(nrows, -1, dtype=np.int64)
    row_weight = np.zeros(nrows, dtype=np.float32)
    row_pair = np.full(nrows, -1, dtype=np.int64)
    pair_row = np.full(P, -1, dtype=np.int64)
    tile_group = np.zeros(num_tiles, dtype=np.int64)
    pos = 0
    for g in range(n_groups):
        sel = order[pos:pos + counts[g]]
        pos += counts[g]
        r = offsets[g] + np.arange(counts[g])
        row_token[r] = t_of[sel]
        row_tenant[r] = lora_tenant[sel]
        row_weight[r] = wt[sel]
        row_pair[r] = sel
        pair_row[sel] = r
        tile_group[offsets[g] // 128: offsets[g + 1] // 128] = g
    return {"row_token": row_token, "row_tenant": row_tenant, "row_weight": row_weight, "row_pair": row_pair,
            "pair_row": pair_row, "tile_group": tile_group, "group_offsets": offsets, "group_counts": counts,
            "num_tiles": num_tiles, "dropped": int(bad.sum())}
