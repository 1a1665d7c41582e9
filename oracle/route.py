"""Router restatement (test infrastructure).

make_routing (benchmarks/real_moe_lora_residual_bench.py:360-386):
  logits = float32(x) @ W_g^T;  weights, ids = topk(softmax(logits), k)
followed by normalize_routing_weights (stageml/moe_lora_layers.py:178-183):
  weights / max(sum(weights), 1e-12).
Selection is made on the logits (softmax is monotonic), larger first, ties to
the lower expert index; this equals the reference's selection on the fp32
probabilities except where rounding makes two different logits' probabilities
equal, where the reference's tie order is torch.topk's.
"""

from __future__ import annotations

import numpy as np


def router_logits(x: np.ndarray, gate_w: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32) @ np.asarray(gate_w, dtype=np.float32).T


def softmax(logits: np.ndarray) -> np.ndarray:
    l64 = np.asarray(logits, dtype=np.float64)
    m = l64.max(axis=-1, keepdims=True)
    e = np.exp(l64 - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def topk_ids(logits: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest logits per row, larger first, ties -> lower index."""
    l = np.asarray(logits, dtype=np.float32)
    T, E = l.shape
    # lexsort: last key is primary -> sort by (-logit, index)
    order = np.lexsort((np.broadcast_to(np.arange(E), (T, E)), -l), axis=-1)
    return order[:, :k].astype(np.int64)


def topk_from_logits(logits: np.ndarray, k: int, renormalize: bool = True) -> tuple[np.ndarray, np.ndarray]:
    probs = softmax(logits)
    ids = topk_ids(logits, k)
    w = np.take_along_axis(probs, ids, axis=-1).astype(np.float32)
    if renormalize:
        w = normalize_routing_weights(w)
    return ids, w


def normalize_routing_weights(w: np.ndarray) -> np.ndarray:
    w = np.asarray(w, dtype=np.float32)
    denom = np.maximum(w.sum(axis=1, keepdims=True), np.float32(1e-12))
    return (w / denom).astype(np.float32)


def route_topk(x: np.ndarray, gate_w: np.ndarray, k: int, renormalize: bool = True):
    """-> (ids int64 [T,k], weights fp32 [T,k], logits fp32 [T,E])."""
    logits = router_logits(x, gate_w)
    ids, w = topk_from_logits(logits, k, renormalize)
    return ids, w, logits
