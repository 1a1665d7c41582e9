"""Folded weight sets served beside dynamic adapters in one MoE layer call.

The reference decides per (adapter, expert) whether an adapter's residual is
folded into the expert's weights at stage 0 (``materialized_residual`` entries of
``choose_residual_plan``, stageml/residual_planner.py:48-153; ``RequestExecutor``'s
materialized adapters, benchmarks/multitenant_bta_system_bench.py:389-396) and
then serves folded tenants and dynamic tenants through separate calls
(``bta_one`` vs ``dynamic_one``, and the split of stageml/vllm_stage_router.py:138-157).

Here the folded sets live after the base experts in one ``gate_up`` bank
``[E + F, 2I, H]``; ``fold_slot[a, e]`` names the set of (adapter a, expert e) or
-1, and ``down_group`` maps every weight group to its down projection (folded w1
adapters leave w2 unchanged, so a folded set reads its base expert's ``down``).
``stageml_moe_forward`` takes all three and routes each (token, expert) pair to
its weight group inside the permutation: one call, no host read, no sub-batches.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops

__all__ = ["FoldedWeightSets", "fold_w1_sets"]


@dataclass
class FoldedWeightSets:
    gate_up: torch.Tensor     # [E + F, 2I, H]: base experts, then the folded sets
    down: torch.Tensor        # [E, H, I]: base experts only
    fold_slot: torch.Tensor   # [n_adapters, E] int32 (-1 = dynamic)
    down_group: torch.Tensor  # [E + F] int32: down projection of each weight group
    n_fold: int
    slots: dict               # (adapter, expert) -> slot

    @property
    def num_experts(self) -> int:
        return int(self.down.shape[0])

    def base_gate_up(self) -> torch.Tensor:
        return self.gate_up[: self.num_experts]

    def adapter_gate_up(self, adapter: int) -> torch.Tensor | None:
        """The adapter's folded sets as a contiguous [E, 2I, H] view when it is folded into
        every expert in expert order (the residual gate_up of bta_one), else None."""
        E = self.num_experts
        s = [self.slots.get((adapter, e)) for e in range(E)]
        if any(v is None for v in s) or s != list(range(s[0], s[0] + E)):
            return None
        return self.gate_up[E + s[0]: E + s[0] + E]

    def moe_kwargs(self) -> dict:
        """Keyword arguments of ops.moe_forward that select the folded sets."""
        if self.n_fold == 0:
            return {}
        return {"fold_slot": self.fold_slot, "n_fold": self.n_fold, "down_group": self.down_group}


def fold_w1_sets(gate_up: torch.Tensor, down: torch.Tensor, adapters, folds) -> FoldedWeightSets:
    """Fold w1 adapters into copies of their experts' gate_up rows at stage 0, on the device.

    adapters: objects with ``A [E, r, H]``, ``B [E, I, r]`` and ``scaling`` (MoEAdapterSpec);
    folds: (adapter index, expert ids) pairs; set (a, e) = gate_up[e] with rows [:I]
    replaced by W1_e + s_a B_a,e A_a,e (the fold of MaterializedMoELoRALayer.__init__,
    stageml/moe_lora_layers.py:104-110), rows [I:] unchanged.
    """
    E, I2, H = (int(v) for v in gate_up.shape)
    I = I2 // 2
    dev, dt = gate_up.device, gate_up.dtype
    F = sum(len(ex) for _, ex in folds)
    bank = torch.empty((E + F, I2, H), dtype=dt, device=dev)
    bank[:E].copy_(gate_up)
    fold_slot = torch.full((len(adapters), E), -1, dtype=torch.int32)
    down_group = list(range(E))
    slots: dict = {}
    s = 0
    for a, experts in folds:
        ex = [int(e) for e in experts]
        if any(not 0 <= e < E for e in ex):
            raise ValueError(f"fold of adapter {a} names expert ids outside [0, {E})")
        if not ex:
            continue
        ad = adapters[a]
        idx = torch.tensor(ex, device=dev)
        n = len(ex)
        bank[E + s: E + s + n, :I] = ops.lora_fold(gate_up[idx, :I].contiguous(), ad.A[idx].to(dev, dt),
                                                   ad.B[idx].to(dev, dt), float(ad.scaling))
        bank[E + s: E + s + n, I:] = gate_up[idx, I:]
        for j, e in enumerate(ex):
            fold_slot[a, e] = s + j
            slots[(a, e)] = s + j
        down_group += ex
        s += n
    return FoldedWeightSets(gate_up=bank, down=down.contiguous(), fold_slot=fold_slot.to(dev),
                            down_group=torch.tensor(down_group, dtype=torch.int32, device=dev), n_fold=F,
                            slots=slots)
