"""Expert-parallel MoE-LoRA layer (one process per GPU).

Rank g of N owns routed experts [g*E/N, (g+1)*E/N) together with their slices
of the LoRA banks (adapter factors live with their experts), plus a replica of
every always-on shared expert. One layer call:

  1. route the rank's own tokens (fp32 router, top-k, renormalise);
  2. send every routed (token, slot) pair -- the row of x and its (local expert,
     tenant, routing weight) -- to the rank owning its expert;
  3. run the received rows through the local grouped SwiGLU experts with LoRA
     (stageml_moe_forward with one expert per row and the routing weight
     applied in the down-projection epilogue);
  4. send the outputs back and combine them per token with the shared experts'
     output computed locally.

Two transports. "peer" (default on CUDA with NCCL): steps 2 and 4 are the C
ABI's stageml_ep_dispatch / stageml_ep_return / stageml_ep_combine -- stores
into the other GPUs' memory through CUDA IPC mappings over NVLink with epoch
flags, so the host never waits for split sizes. "collective": all_to_all_single
of counts, rows and packed records, and back (any backend; with route, local
compute and combine injectable, the host logic runs with gloo on CPU).

The reference has no distributed code; this is the expert-parallel layout of
the path. All ranks make the same calls in the same order, also when a rank
sends or receives nothing.

The layer is also a torch op, ``torch.ops.stageml.ep_moe_lora_forward(x,
tenant_ids, layer)``, with ``layer`` the handle ``EPMoELayer.register()``
returns: the same call through the dispatcher (CUDA key only, a fake
implementation for tracing), beside the single-GPU ``stageml::moe_forward``.
"""

from __future__ import annotations

from typing import Callable, Optional

import ctypes

import torch
import torch.distributed as dist


class EPMoELayer:
    def __init__(self, *, E: int, k: int, n_shared: int, H: int, I: int, rank: int, world: int,
                 gate_up_local: torch.Tensor, down_local: torch.Tensor, router_w: torch.Tensor, n_tenants: int = 0,
                 lora_rank: int = 0, lora_a13=None, lora_b13=None, lora_a2=None, lora_b2=None, lora_scale=None,
                 group=None, route_fn: Optional[Callable] = None, local_fn: Optional[Callable] = None,
                 shared_fn: Optional[Callable] = None, combine_fn: Optional[Callable] = None,
                 transport: str = "auto", max_tokens: Optional[int] = None):
        if E % world:
            raise ValueError(f"{E} routed experts do not split evenly over {world} ranks")
        if transport not in ("auto", "peer", "collective"):
            raise ValueError(f"unknown transport {transport!r}")
        self.E, self.k, self.n_shared, self.H, self.I = E, k, n_shared, H, I
        self.rank, self.world, self.group = rank, world, group
        self.E_loc = E // world
        self.gate_up, self.down, self.router_w = gate_up_local, down_local, router_w
        self.n_tenants, self.lora_rank = n_tenants, lora_rank
        self.lora = dict(lora_a13=lora_a13, lora_b13=lora_b13, lora_a2=lora_a2, lora_b2=lora_b2)
        self.lora_scale = lora_scale
        injected = any(f is not None for f in (route_fn, local_fn, shared_fn, combine_fn))
        self.route_fn = route_fn or self._route
        self.local_fn = local_fn or self._local
        self.shared_fn = shared_fn or self._shared
        self.combine_fn = combine_fn or self._combine
        if transport == "auto":
            on_nccl = dist.is_initialized() and dist.get_backend(group) == "nccl"
            transport = "peer" if (on_nccl and not injected and torch.cuda.is_available()) else "collective"
        if transport == "peer" and injected:
            raise ValueError("the peer transport runs the CUDA route / local / combine steps; do not inject them")
        self.transport = transport
        self.max_tokens = max_tokens
        self._peer = None

    # ------------------------------------------------------------ factories
    @classmethod
    def from_full_weights(cls, cfg, w: dict, *, rank: int, world: int, group=None, transport: str = "auto",
                          max_tokens: Optional[int] = None) -> "EPMoELayer":
        """Slice a full set of layer weights (layout of stageml_b200.workloads.make_moe_workload) for one rank."""
        E_loc = cfg.E // world
        own = list(range(rank * E_loc, (rank + 1) * E_loc)) + list(range(cfg.E, cfg.E + cfg.n_shared))
        idx = torch.tensor(own, device=w["gate_up"].device)
        take = lambda t, d: None if t is None else t.index_select(d, idx).contiguous()
        return cls(E=cfg.E, k=cfg.k, n_shared=cfg.n_shared, H=cfg.H, I=cfg.I, rank=rank, world=world,
                   gate_up_local=take(w["gate_up"], 0), down_local=take(w["down"], 0), router_w=w["router_w"],
                   n_tenants=cfg.n_tenants, lora_rank=cfg.bank_rank, lora_a13=take(w["lora_a13"], 1),
                   lora_b13=take(w["lora_b13"], 1), lora_a2=take(w["lora_a2"], 1), lora_b2=take(w["lora_b2"], 1),
                   lora_scale=w["lora_scale"], group=group, transport=transport, max_tokens=max_tokens)

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
                               topk_weights=weight[:, None].contiguous(),
                               tenant_ids=tenant.contiguous() if self.lora_rank else None, **self._lora_kw())

    def _shared(self, x, tenant):
        from . import ops

        return ops.moe_forward(x, self.gate_up, self.down, k=0, n_shared=self.n_shared,
                               tenant_ids=tenant if self.lora_rank else None, **self._lora_kw())

    @staticmethod
    def _combine(y_back, pair_row, T, k):
        from . import ops

        return ops.combine_rows(y_back, pair_row, T, k)

    # ------------------------------------------------------------ forward
    def __call__(self, x: torch.Tensor, tenant_ids: torch.Tensor) -> torch.Tensor:
        if self.transport == "peer":
            return self._forward_peer(x, tenant_ids)
        return self._forward_collective(x, tenant_ids)

    def _forward_collective(self, x: torch.Tensor, tenant_ids: torch.Tensor) -> torch.Tensor:
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

    # ------------------------------------------------------------ peer-memory transport
    def _setup_peer(self, x: torch.Tensor) -> None:
        """Collective, once: size the exchange buffers for the largest batch of any rank,
        allocate this rank's workspace and map every other rank's through CUDA IPC."""
        from . import capi as C
        from ._native import load_capi

        lib = load_capi()
        dev = x.device
        cap = self.max_tokens
        if cap is None:
            t = torch.tensor([x.shape[0]], dtype=torch.int64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            cap = int(t.item())
        dtype = C.BF16 if x.dtype == torch.bfloat16 else C.F16
        L = C.EpLayout()
        C.check(lib, lib.stageml_ep_get_layout(self.world, cap, self.k, self.H, dtype, ctypes.byref(L)), "ep layout")
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        C.check(lib, lib.stageml_ep_workspace_alloc(L.total, ctypes.byref(base), handle), "ep workspace")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        bases, opened = [], []
        for r in range(self.world):
            if r == self.rank:
                bases.append(base.value)
                continue
            h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
            p = ctypes.c_void_p()
            C.check(lib, lib.stageml_ep_workspace_open(h, ctypes.byref(p)), "ep open")
            bases.append(p.value)
            opened.append(p.value)
        recv_cap = self.world * cap * self.k

        def view(off, shape, typestr, torch_dtype=None):
            cai = {"shape": tuple(shape), "typestr": typestr, "data": (base.value + off, False), "version": 3}
            t = torch.as_tensor(type("_Dev", (), {"__cuda_array_interface__": cai})(), device=dev)
            return t.view(torch_dtype) if torch_dtype is not None else t

        self._peer = dict(
            lib=lib, layout=L, base=base.value, opened=opened, cap=cap, dtype=dtype,
            peers=torch.tensor(bases, dtype=torch.int64, device=dev),
            recv_x=view(L.recv_x, (recv_cap, self.H), "<i2", x.dtype),
            recv_expert=view(L.recv_expert, (recv_cap, 1), "<i4"),
            recv_weight=view(L.recv_weight, (recv_cap, 1), "<f4"),
            recv_tenant=view(L.recv_tenant, (recv_cap,), "<i4"),
            recv_tokens=view(L.recv_tokens, (1,), "<i4"),
            pos=torch.empty(cap * self.k, dtype=torch.int32, device=dev),
            status=torch.zeros(1, dtype=torch.int32, device=dev),
            epoch=0)

    def _forward_peer(self, x: torch.Tensor, tenant_ids: torch.Tensor) -> torch.Tensor:
        from . import capi as C
        from . import ops

        if self._peer is None:
            self._setup_peer(x)
        pe = self._peer
        T = x.shape[0]
        if T > pe["cap"]:
            raise ValueError(f"{T} tokens exceed the {pe['cap']} the exchange buffers were sized for (max_tokens)")
        ids, wts = self.route_fn(x)
        ids = ids.to(torch.int32).contiguous()
        wts = wts.to(torch.float32).contiguous()
        ten = tenant_ids.to(torch.int32).contiguous() if tenant_ids is not None else None
        pe["epoch"] += 1
        a = C.EpArgs(world=self.world, rank=self.rank, T=T, k=self.k, H=self.H, E_loc=self.E_loc,
                     act_dtype=pe["dtype"], epoch=pe["epoch"], tokens_cap=pe["cap"], timeout_ns=0,
                     peers=pe["peers"].data_ptr(), self=pe["base"], topk_ids=ids.data_ptr(),
                     topk_weights=wts.data_ptr(), tenant_ids=C.ptr(ten), x=x.contiguous().data_ptr(),
                     pos=pe["pos"].data_ptr(), status=pe["status"].data_ptr())
        lib, stream = pe["lib"], C.stream_handle()
        C.check(lib, lib.stageml_ep_dispatch(ctypes.byref(a), stream), "ep dispatch")
        y_local = ops.moe_forward(pe["recv_x"], self.gate_up, self.down, topk_ids=pe["recv_expert"],
                                  topk_weights=pe["recv_weight"],
                                  tenant_ids=pe["recv_tenant"] if self.lora_rank else None,
                                  T_dev=pe["recv_tokens"], **self._lora_kw())
        C.check(lib, lib.stageml_ep_return(ctypes.byref(a), y_local.data_ptr(), stream), "ep return")
        shared = self.shared_fn(x, tenant_ids) if self.n_shared else None
        out = torch.empty_like(x)
        C.check(lib, lib.stageml_ep_combine(ctypes.byref(a), C.ptr(shared), out.data_ptr(), stream), "ep combine")
        return out

    def register(self) -> int:
        """Handle of this layer for torch.ops.stageml.ep_moe_lora_forward (valid until close())."""
        for h, layer in _EP_LAYERS.items():
            if layer is self:
                return h
        h = max(_EP_LAYERS, default=0) + 1
        _EP_LAYERS[h] = self
        return h

    def take_status(self) -> int:
        """Device status word of the exchange (synchronises); 0 when every call completed."""
        if self._peer is None:
            return 0
        v = int(self._peer["status"].item())
        self._peer["status"].zero_()
        return v

    def close(self) -> None:
        """Collective: unmap the other ranks' workspaces and free this rank's (after a barrier)."""
        for h in [h for h, layer in _EP_LAYERS.items() if layer is self]:
            del _EP_LAYERS[h]
        if self._peer is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = self._peer["lib"]
        for p in self._peer["opened"]:
            lib.stageml_ep_workspace_close(p)
        dist.barrier(group=self.group)
        lib.stageml_ep_workspace_free(self._peer["base"])
        self._peer = None


# ------------------------------------------------------------ the torch op
_EP_LAYERS: dict = {}


def _define_op() -> None:
    from . import ops  # noqa: F401  (loads the stageml op library first)

    lib = torch.library.Library("stageml", "FRAGMENT")
    lib.define("ep_moe_lora_forward(Tensor x, Tensor tenant_ids, int layer) -> Tensor")

    def impl(x, tenant_ids, layer):
        ep = _EP_LAYERS.get(int(layer))
        if ep is None:
            raise RuntimeError(f"ep_moe_lora_forward: no expert-parallel layer registered as {layer}")
        return ep(x, tenant_ids)

    lib.impl("ep_moe_lora_forward", impl, "CUDA")

    @torch.library.register_fake("stageml::ep_moe_lora_forward")
    def _(x, tenant_ids, layer):
        return x.new_empty(x.shape)

    globals()["_OP_LIB"] = lib  # the registration lives as long as the library object


try:
    _define_op()
except RuntimeError as exc:  # pragma: no cover - defined already in this process
    if "already" not in str(exc):
        raise


__all__ = ["EPMoELayer"]
