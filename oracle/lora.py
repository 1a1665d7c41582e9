"""Dense LoRA restatements in numpy (test infrastructure).

lora_fold             W + s * B @ A ([out,in]) -- materialize_residual_weight
                      (stageml/triton_generator.py:175-191), StageMLAdapterBankLinear.__init__
                      (stageml/adapter_bank.py:90-94), MaterializedMoELoRALayer.__init__
                      (stageml/moe_lora_layers.py:104-110); or W + s * A @ B ([in,out], the
                      folded single LoRA of benchmarks/triton_lora_equivalence_check.py:11-22)
dynamic_lora_linear   DynamicLoRALinear.forward (stageml/adapter_bank.py:58-69)
adapter_bank_linear   StageMLAdapterBankLinear.forward (stageml/adapter_bank.py:101-109)
cost_based_cache      StageMLCostBasedAdapterCache.forward (stageml/adapter_cache.py:83-100)
choose_hot_adapters   stageml/adapter_cache.py:106-140
single_lora           y = x W + s (x A) B, W [in,out] (benchmarks/triton_lora_equivalence_check.py:11-12)
"""

from __future__ import annotations

import numpy as np


def lora_fold(W, A, B, scale, layout: int = 0, dtype=np.float64):
    W = np.asarray(W, dtype=dtype)
    A = np.asarray(A, dtype=dtype)
    B = np.asarray(B, dtype=dtype)
    if layout == 0:
        return W + dtype(scale) * (B @ A)
    return W + dtype(scale) * (A @ B)


def dynamic_lora_linear(x, W, bias, A, B, scale, row_adapter, dtype=np.float64):
    """A [n, r, K], B [n, N, r], scale [n]; row_adapter[m] in [0, n) (every row has an adapter)."""
    x = np.asarray(x, dtype=dtype)
    y = x @ np.asarray(W, dtype=dtype).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=dtype)
    ra = np.asarray(row_adapter, dtype=np.int64)
    for a in np.unique(ra):
        m = ra == a
        y[m] += dtype(scale[a]) * ((x[m] @ np.asarray(A[a], dtype=dtype).T) @ np.asarray(B[a], dtype=dtype).T)
    return y


def adapter_bank_linear(x, merged, bias, row_adapter, dtype=np.float64):
    x = np.asarray(x, dtype=dtype)
    ra = np.asarray(row_adapter, dtype=np.int64)
    y = np.zeros((x.shape[0], merged.shape[1]), dtype=dtype)
    for a in np.unique(ra):
        m = ra == a
        y[m] = x[m] @ np.asarray(merged[a], dtype=dtype).T
    if bias is not None:
        y = y + np.asarray(bias, dtype=dtype)
    return y


def cost_based_cache(x, W, bias, A, B, scale, cached: list[int], row_adapter, dtype=np.float64):
    """Rows of cached adapters use W + s B A, the others the dynamic form."""
    x = np.asarray(x, dtype=dtype)
    ra = np.asarray(row_adapter, dtype=np.int64)
    y = np.zeros((x.shape[0], W.shape[0]), dtype=dtype)
    for a in np.unique(ra):
        m = ra == a
        if int(a) in cached:
            Wp = lora_fold(W, A[a], B[a], scale[a], 0, dtype)
            y[m] = x[m] @ Wp.T
        else:
            y[m] = x[m] @ np.asarray(W, dtype=dtype).T + dtype(scale[a]) * (
                (x[m] @ np.asarray(A[a], dtype=dtype).T) @ np.asarray(B[a], dtype=dtype).T)
        if bias is not None:
            y[m] += np.asarray(bias, dtype=dtype)
    return y


def choose_hot_adapters(request_counts: dict, names: list[str], *, in_features: int, out_features: int,
                        bytes_per_weight: int, memory_budget_mb: float) -> list[str]:
    per = in_features * out_features * bytes_per_weight
    budget = int(memory_budget_mb * 1024 * 1024)
    ranked = sorted(names, key=lambda n: (-int(request_counts.get(n, 0)), n))
    cached, used = [], 0
    for n in ranked:
        if used + per <= budget and int(request_counts.get(n, 0)) > 0:
            cached.append(n)
            used += per
    return cached


def single_lora(x, W, A, B, scale, dtype=np.float64):
    x = np.asarray(x, dtype=dtype)
    y = x @ np.asarray(W, dtype=dtype)
    if A is not None:
        y = y + dtype(scale) * ((x @ np.asarray(A, dtype=dtype)) @ np.asarray(B, dtype=dtype))
    return y
