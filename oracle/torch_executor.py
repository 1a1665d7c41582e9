"""The reference's request executor restated with torch CPU ops (test infrastructure).

Follows RequestExecutor.dynamic_one (benchmarks/multitenant_bta_system_bench.py:398-414)
operation by operation: for each top-k slot and each expert, torch.nonzero picks the
rows routed there, index_select gathers them, F.linear applies w1 (plus the LoRA term
s * (x A^T) B^T) and w3, silu(w1 path) * (w3 path) goes through F.linear with w2, and
index_add_ accumulates the rows weighted by their routing weight. The reference serves
one adapter per call; a batch with per-token tenants is the sum of its requests' calls,
so here each (slot, expert) group applies every tenant's adapter to that tenant's
rows. LoRA on w3 and w2 (when given) is the same term, as DynamicMoELoRALayer.forward
applies it (stageml/moe_lora_layers.py:85-89); always-on shared experts follow the
routed slots with weight 1.

Used as the timed CPU baseline of the benchmark (the torch CPU execution the
reference's executor performs) and checked against the reference's own outputs
(tests/golden/request_executor.npz). Never part of the product path.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


@torch.no_grad()
def dynamic_executor(x, gate_up, down, ids, weights, tenant_ids=None, *, n_shared: int = 0, lora_a13=None,
                     lora_b13=None, lora_a2=None, lora_b2=None, lora_scale=None) -> torch.Tensor:
    """out [T, H]; layouts as the C ABI (gate_up [E_tot, 2I, H] with rows [:I] = w1, down [E_tot, H, I],
    lora_a13 [nT, E_tot, 2r, H], lora_b13 [nT, E_tot, 2I, r], lora_a2 [nT, E_tot, r, I],
    lora_b2 [nT, E_tot, H, r]); tenant -1 = no adapter."""
    T = x.shape[0]
    E_tot = gate_up.shape[0]
    I = gate_up.shape[1] // 2
    E = E_tot - n_shared
    w1, w3 = gate_up[:, :I], gate_up[:, I:]
    r = 0 if lora_a13 is None else lora_a13.shape[2] // 2
    ten = torch.full((T,), -1, dtype=torch.int64) if tenant_ids is None else tenant_ids.to(torch.int64)
    out = torch.zeros((T, down.shape[1]), dtype=x.dtype)
    slots = [(ids[:, j], weights[:, j].to(x.dtype)) for j in range(ids.shape[1])]
    slots += [(torch.full((T,), E + s, dtype=torch.int64), torch.ones(T, dtype=x.dtype)) for s in range(n_shared)]
    for eids, gates in slots:
        for expert in range(E_tot):
            index = torch.nonzero(eids == expert, as_tuple=False).flatten()
            if index.numel() == 0:
                continue
            xs = x.index_select(0, index)
            up = F.linear(xs, w1[expert])
            gate = F.linear(xs, w3[expert])
            tn = ten.index_select(0, index)
            tenants = torch.unique(tn[tn >= 0]).tolist() if lora_a13 is not None or lora_a2 is not None else []
            for a in tenants:
                m = torch.nonzero(tn == a, as_tuple=False).flatten()
                xa = xs.index_select(0, m)
                if lora_a13 is not None:
                    s = lora_scale[a]
                    up.index_add_(0, m, s * (xa @ lora_a13[a, expert, :r].t() @ lora_b13[a, expert, :I].t()))
                    gate.index_add_(0, m, s * (xa @ lora_a13[a, expert, r:].t() @ lora_b13[a, expert, I:].t()))
            h = F.silu(up) * gate
            y = F.linear(h, down[expert])
            if lora_a2 is not None:
                for a in tenants:
                    m = torch.nonzero(tn == a, as_tuple=False).flatten()
                    y.index_add_(0, m, lora_scale[a] * (h.index_select(0, m) @ lora_a2[a, expert].t()
                                                        @ lora_b2[a, expert].t()))
            out.index_add_(0, index, y * gates.index_select(0, index).unsqueeze(1))
    return out
