"""MoE-LoRA layer restatements in numpy (test infrastructure).

moe_forward: the SwiGLU expert MLP with per-tenant LoRA of
RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:398-414):
  for each (slot, expert) group: lora = s * (xs @ A[e].T) @ B[e].T
  up = xs @ w1[e].T + lora ; gate = xs @ w3[e].T ; y = (silu(up) * gate) @ down[e].T
  out.index_add_(index, y * weight)
(the reference names gate_up[:, :I] "w1"/"up" and feeds it to SiLU). The same
LoRA term is applied to w3 and w2 when their factors are given, as
DynamicMoELoRALayer.forward does for its single linear
(stageml/moe_lora_layers.py:85-89) -- the reference has no code for LoRA on
w3/w2. Always-on shared experts (n_shared > 0) use expert ids E..E+n_shared-1
and weight 1; the reference has no shared-expert code either.
With no LoRA this is _fallback_moe (stageml/custom_op_registry.py:23-37).

moe_linear: DynamicMoELoRALayer.forward / MaterializedMoELoRALayer.forward
(stageml/moe_lora_layers.py:63-90, 117-142) in grouped form.
"""

from __future__ import annotations

import numpy as np


def silu(v: np.ndarray) -> np.ndarray:
    return v / (1.0 + np.exp(-v))


def _pairs(ids, weights, n_shared, E_routed):
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    cols_e = [ids[:, j] for j in range(k)] + [np.full(T, E_routed + s, dtype=np.int64) for s in range(n_shared)]
    if weights is None:
        cols_w = [np.ones(T) for _ in range(k + n_shared)]
    else:
        w = np.asarray(weights, dtype=np.float64)
        cols_w = [w[:, j] for j in range(k)] + [np.ones(T) for _ in range(n_shared)]
    return cols_e, cols_w


def moe_forward(x, gate_up, down, ids, weights, *, tenant_ids=None, n_shared: int = 0, lora_a13=None, lora_b13=None,
                lora_a2=None, lora_b2=None, lora_scale=None, dtype=np.float64, round_h=None, fold_slot=None,
                down_group=None):
    """out[T,H] of one MoE-LoRA FFN layer.

    Layouts: gate_up [E_tot, 2I, H] (rows [:I] = SiLU branch), down [E_tot, H, I],
    lora_a13 [nT, E_tot, 2r, H] (rows [:r] for gate_up[:, :I]), lora_b13 [nT, E_tot, 2I, r],
    lora_a2 [nT, E_tot, r, I], lora_b2 [nT, E_tot, H, r], lora_scale [nT]; tenant -1 = no adapter.
    round_h: optional function applied to the SwiGLU output before the down projection
    (models the 16-bit intermediate of the device path).
    fold_slot [nT, E_tot]: with it, gate_up / down hold E_tot + n_fold weight groups and a pair
    of tenant a routed to expert e with fold_slot[a, e] = s >= 0 uses group E_tot + s (the
    adapter folded into that expert's weights, as MaterializedMoELoRALayer and the
    residual planner's materialized entries do) without the dynamic LoRA term.
    down_group [E_tot + n_fold]: group g's down projection is down[down_group[g]].
    """
    x = np.asarray(x, dtype=dtype)
    gate_up = np.asarray(gate_up)
    down = np.asarray(down)
    T, H = x.shape
    I = gate_up.shape[1] // 2
    ten = np.full(T, -1, dtype=np.int64) if tenant_ids is None else np.asarray(tenant_ids, dtype=np.int64)
    E_tot = gate_up.shape[0] if fold_slot is None else np.asarray(fold_slot).shape[1]
    E_routed = E_tot - n_shared
    cols_e, cols_w = _pairs(ids, weights, n_shared, E_routed)
    cols_t = [ten for _ in cols_e]  # LoRA tenant of each pair
    if fold_slot is not None:
        fs = np.asarray(fold_slot, dtype=np.int64)
        folded = [np.where(ten >= 0, fs[np.maximum(ten, 0), ce], -1) for ce in cols_e]
        cols_e = [np.where(f >= 0, E_tot + f, ce) for ce, f in zip(cols_e, folded)]
        cols_t = [np.where(f >= 0, -1, ten) for f in folded]
    out = np.zeros((T, H), dtype=dtype)
    r = 0 if lora_a13 is None and lora_a2 is None else (
        lora_a13.shape[2] // 2 if lora_a13 is not None else lora_a2.shape[2])
    for e in range(gate_up.shape[0]):
        rows_list = [np.nonzero(ce == e)[0] for ce in cols_e]
        idx = np.concatenate(rows_list)
        if idx.size == 0:
            continue
        wgt = np.concatenate([cw[rl] for cw, rl in zip(cols_w, rows_list)]).astype(dtype)
        xs = x[idx]
        w13 = gate_up[e].astype(dtype)
        gu = xs @ w13.T
        tn = np.concatenate([ct[rl] for ct, rl in zip(cols_t, rows_list)])
        if lora_a13 is not None:
            for a in np.unique(tn[tn >= 0]):
                m = tn == a
                s = (xs[m] @ np.asarray(lora_a13[a, e], dtype=dtype).T) * dtype(lora_scale[a])
                b = np.asarray(lora_b13[a, e], dtype=dtype)
                gu[m, :I] += s[:, :r] @ b[:I].T
                gu[m, I:] += s[:, r:] @ b[I:].T
        h = silu(gu[:, :I]) * gu[:, I:]
        if round_h is not None:
            h = round_h(h).astype(dtype)
        y = h @ down[e if down_group is None else int(down_group[e])].astype(dtype).T
        if lora_a2 is not None:
            for a in np.unique(tn[tn >= 0]):
                m = tn == a
                s2 = (h[m] @ np.asarray(lora_a2[a, e], dtype=dtype).T) * dtype(lora_scale[a])
                y[m] += s2 @ np.asarray(lora_b2[a, e], dtype=dtype).T
        contrib = y * wgt[:, None]
        if np.unique(idx).size == idx.size:
            out[idx] += contrib
        else:  # a token routed twice to the same expert
            np.add.at(out, idx, contrib)
    return out


def fallback_moe(hidden, gate_up, down, topk_weights, topk_ids, dtype=np.float64):
    """_fallback_moe (stageml/custom_op_registry.py:23-37): the residual_moe op's semantics."""
    return moe_forward(hidden, gate_up, down, topk_ids, topk_weights, dtype=dtype)


def moe_linear(x, weight, ids, weights, *, bias=None, tenant_ids=None, lora_a=None, lora_b=None, lora_scale=None,
               merged=None, dtype=np.float64):
    """Routed single linear: out[t] = sum_j w[t,j] (x_t W[e]^T + b[e] + s_a (x_t A[a,e]^T) B[a,e]^T).

    weight [E, N, K]; lora_a [nT, E, r, K]; lora_b [nT, E, N, r]; merged [nA, E, N, K] selects
    merged[a, e] instead (MaterializedMoELoRALayer), in which case LoRA is not added.
    """
    x = np.asarray(x, dtype=dtype)
    ids = np.asarray(ids, dtype=np.int64)
    T, k = ids.shape
    N = weight.shape[1] if merged is None else merged.shape[2]
    out = np.zeros((T, N), dtype=dtype)
    ten = None if tenant_ids is None else np.asarray(tenant_ids, dtype=np.int64)
    w = np.asarray(weights, dtype=dtype)
    for j in range(k):
        e = ids[:, j]
        if merged is not None:
            Wt = np.asarray(merged, dtype=dtype)[ten, e]
        else:
            Wt = np.asarray(weight, dtype=dtype)[e]
        y = np.einsum("tk,tnk->tn", x, Wt)
        if bias is not None:
            y += np.asarray(bias, dtype=dtype)[e]
        if merged is None and lora_a is not None:
            A = np.asarray(lora_a, dtype=dtype)[ten, e]
            B = np.asarray(lora_b, dtype=dtype)[ten, e]
            s = np.einsum("tk,trk->tr", x, A) * np.asarray(lora_scale, dtype=dtype)[ten][:, None]
            y += np.einsum("tr,tnr->tn", s, B)
        out += w[:, j:j + 1] * y
    return out


class MoEExecutorF32:
    """float32 grouped executor over host weights, used as the timed CPU baseline.

    Same math as moe_forward; weights are converted once (stage 0) and each call
    runs one BLAS GEMM per (expert, projection) plus per-tenant LoRA GEMMs.
    """

    def __init__(self, gate_up, down, *, n_shared=0, lora_a13=None, lora_b13=None, lora_a2=None, lora_b2=None,
                 lora_scale=None):
        self.gate_up = np.ascontiguousarray(gate_up, dtype=np.float32)
        self.down = np.ascontiguousarray(down, dtype=np.float32)
        self.n_shared = n_shared
        self.lora_a13 = None if lora_a13 is None else np.ascontiguousarray(lora_a13, dtype=np.float32)
        self.lora_b13 = None if lora_b13 is None else np.ascontiguousarray(lora_b13, dtype=np.float32)
        self.lora_a2 = None if lora_a2 is None else np.ascontiguousarray(lora_a2, dtype=np.float32)
        self.lora_b2 = None if lora_b2 is None else np.ascontiguousarray(lora_b2, dtype=np.float32)
        self.lora_scale = None if lora_scale is None else np.asarray(lora_scale, dtype=np.float32)

    def __call__(self, x, ids, weights, tenant_ids=None):
        return moe_forward(x, self.gate_up, self.down, ids, weights, tenant_ids=tenant_ids, n_shared=self.n_shared,
                           lora_a13=self.lora_a13, lora_b13=self.lora_b13, lora_a2=self.lora_a2,
                           lora_b2=self.lora_b2, lora_scale=self.lora_scale, dtype=np.float32)
