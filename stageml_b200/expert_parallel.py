"""Expert-parallel MoE-LoRA layer over NCCL (one process per GPU).

Rank g of N owns routed experts [g*E/N, (g+1)*E/N) together with their slices
of the LoRA banks (adapter factors live with their experts), plus a replica of
every always-on shared expert. One layer call:

  1. route the rank's own tokens (fp32 router, top-k, renormalise);
  2. order the routed (token, slot) pairs by owning rank and exchange counts
     (all_to_all_single of N int64), then rows of x and a packed int32
     (local expert, tenant, routing weight bits) record per pair
     (two all_to_all_single of the uneven splits);
  3. run the received rows through the local grouped SwiGLU experts with LoRA
     (stageml_moe_forward with one expert per row and the routing weight
     applied in the down-projection epilogue);
  4. send the outputs back (all_to_all_single) and combine them per token with
     the shared experts' output computed locally.

The reference has no distributed code; this is the expert-parallel layout the
path's north star asks for. All ranks issue the same collectives in the same
order, also for empty splits. Routing, the local compute and the combine are
injectable so the host logic can be tested with gloo on CPU.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


class EPMoELayer:
    def __init__(self, *, E: int, k: int, n_shared: int, H: int, I: int, rank: int, world: int,
                 gate_up_local: torch.Tensor, down_local: torch.Tensor, router_w: torch.Tensor, n_tenants: int = 0,
                 lora_rank: int = 0, lora_a13=None, lora_b13=None, lora_a2=None, lora_b2=None, lora_scale=None,
                 group=None, route_fn: Optional[Callable] = None, local_fn: Optional[Callable] = None,
                 shared_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None):
        if E % world:
            raise ValueError(f"{E} routed experts do not split evenly over {world} ranks")
        self.E, self.k, self.n_shared, self.H, self.I = E, k, n_shared, H, I
        self.rank, self.world, self.group = rank, world, group
        self.E_loc = E // world
        self.gate_up, self.down, self.router_w = gate_up_local, down_local, router_w
        self.n_tenants, self.lora_rank = n_tenants, lora_rank
        self.lora = dict(lora_a13=lora_a13, lora_b13=lora_b13, lora_a2=lora_a2, lora_b2=lora_b2)
        self.lora_scale = lora_scale
        self.route_fn = route_fn or self._route
        self.local_fn = local_fn or self._local
        self.shared_fn = shared_fn or self._shared
        self.combine_fn = combine_fn or self._combine

    # ------------------------------------------------------------ factories
    @classmethod
    def from_full_weights(cls, cfg, w: dict, *, rank: int, world: int, group=None) -> "EPMoELayer":
        """Slice a full set of layer weights (layout of stageml_b200.workloads.make_moe_workload) for one rank."""
        E_loc = cfg.E // world
        own = list(range(rank * E_loc, (rank + 1) * E_loc)) + list(range(cfg.E, cfg.E + cfg.n_shared))
        idx = torch.tensor(own, device=w["gate_up"].device)
        take = lambda t, d: None if t is None else t.index_select(d, idx).contiguous()
        return cls(E=cfg.E, k=cfg.k, n_shared=cfg.n_shared, H=cfg.H, I=cfg.I, rank=rank, world=world,
                   gate_up_local=take(w["gate_up"], 0), down_local=take(w["down"], 0), router_w=w["router_w"],
                   n_tenants=cfg.n_tenants, lora_rank=cfg.bank_rank, lora_a13=take(w["lora_a13"], 1),
                   lora_b13=take(w["lora_b13"], 1), lora_a2=take(w["lora_a2"], 1), lora_b2=take(w["lora_b2"], 1),
                   lora_scale=w["lora_scale"], group=group)

    # ------------------------------------------------------------ default pieces (CUDA)
    def _route(self, x):
        from . import ops

        ids, wts, _ = ops.route_topk(x, self.router_w, self.k, True)
        return ids, wts

    def _lora_kw(self):
        if not self.lora_rank:
            return {}
        return dict(n_tenants=self.n_tenants, rank=self.lora_rank, lora_scale=self.lora_scale, **self.lora)

    def _local(self, x_recv, expert, tenant, weight):
        from . import ops

        return ops.moe_forward(x_recv, self.gate_up, self.down, topk_ids=expert[:, None].contiguous(),
                               topk_weights=weight[:, None].contiguous(), tenant_ids=tenant.contiguous(),
                               **self._lora_kw())

    def _shared(self, x, tenant):
        from . import ops

        return ops.moe_forward(x, self.gate_up, self.down, k=0, n_shared=self.n_shared, tenant_ids=tenant,
                               **self._lora_kw())

    @staticmethod
    def _combine(y_back, pair_row, T, k):
        from . import ops

        return ops.combine_rows(y_back, pair_row, T, k)

    # ------------------------------------------------------------ forward
    def __call__(self, x: torch.Tensor, tenant_ids: torch.Tensor) -> torch.Tensor:
        T, k, world = x.shape[0], self.k, self.world
        ids, wts = self.route_fn(x)
        flat_ids = ids.reshape(-1).to(torch.int64)
        dest = torch.div(flat_ids, self.E_loc, rounding_mode="floor")
        order = torch.sort(dest, stable=True).indices
        send_counts = torch.bincount(dest, minlength=world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        tok = torch.div(order, k, rounding_mode="floor")
        x_send = x.index_select(0, tok).contiguous()
        meta_send = torch.stack([(flat_ids[order] - dest[order] * self.E_loc).to(torch.int32),
                                 tenant_ids.index_select(0, tok).to(torch.int32),
                                 wts.reshape(-1)[order].to(torch.float32).view(torch.int32)], 1).contiguous()
        n_recv = sum(rc)
        x_recv = x.new_empty((n_recv, x.shape[1]))
        meta_recv = meta_send.new_empty((n_recv, 3))
        dist.all_to_all_single(x_recv, x_send, rc, sc, group=self.group)
        dist.all_to_all_single(meta_recv, meta_send, rc, sc, group=self.group)
        if n_recv:
            y_recv = self.local_fn(x_recv, meta_recv[:, 0].contiguous(), meta_recv[:, 1].contiguous(),
                                   meta_recv[:, 2].contiguous().view(torch.float32))
        else:
            y_recv = x.new_empty((0, x.shape[1]))
        y_back = x.new_empty((T * k, x.shape[1]))
        dist.all_to_all_single(y_back, y_recv.contiguous(), sc, rc, group=self.group)
        pair_row = torch.empty_like(order)
        pair_row[order] = torch.arange(order.numel(), device=order.device)
        out = self.combine_fn(y_back, pair_row.to(torch.int32), T, k)
        if self.n_shared:
            out = out + self.shared_fn(x, tenant_ids)
        return out


__all__ = ["EPMoELayer"]
