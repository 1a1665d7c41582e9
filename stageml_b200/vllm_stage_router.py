"""Tenant router for a vLLM fused-MoE interception point (reference: stageml/vllm_stage_router.py).

Tokens of tenants that have a StageML residual kernel go to the
``stageml::residual_moe`` op (here: the sm_100a grouped GEMM path); the others
go to vLLM's ``fused_experts``. Same classes and functions as the reference.

Difference in the split: the reference moves the tenant ids to the host to
build the mask (``tenant_ids.cpu().tolist()``, stageml/vllm_stage_router.py:60-63).
Here the mask is a device-side table lookup; the host only learns the number
of selected tokens (one scalar) to size the two sub-batches. With
``split="masked"`` there is no host synchronisation at all: both backends see the
whole batch, each with the other backend's routing weights set to zero, and the
two outputs are added (twice the expert work, no host read-back). With
``split="device"`` one call of this package's MoE op serves the whole batch: the
tenant mask stays on the device, tokens of tenants with a kernel run on their
folded weight sets (``weight_sets``, stageml_b200/folded_sets.py) and every other
token on the base experts -- the fused-MoE arithmetic vLLM's ``fused_experts``
performs, in the same launches -- with no host read-back and no doubled work.
"""

from __future__ import annotations

import importlib
import json
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Callable

import torch

from .custom_op_registry import ensure_stageml_custom_op


@dataclass(frozen=True)
class KernelManifestEntry:
    tenant_id: int
    adapter_id: int
    backend: str
    artifact: str
    symbol: str = "stageml_residual_moe"
    enabled: bool = True


@dataclass(frozen=True)
class KernelManifest:
    version: int
    model: str
    entries: tuple[KernelManifestEntry, ...]

    def to_dict(self) -> dict[str, Any]:
        return {"version": self.version, "model": self.model, "entries": [asdict(e) for e in self.entries]}


def read_kernel_manifest(path: str | Path) -> KernelManifest:
    """Tenant -> artifact manifest, JSON format of stageml/baremetal_backend.py:159-193."""
    data = json.loads(Path(path).read_text())
    entries = tuple(KernelManifestEntry(**e) for e in data.get("entries", []))
    return KernelManifest(version=int(data.get("version", 1)), model=str(data.get("model", "unknown")), entries=entries)


def write_kernel_manifest(path: str | Path, manifest: KernelManifest) -> Path:
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(manifest.to_dict(), indent=2, sort_keys=True) + "\n")
    return out


@dataclass(frozen=True)
class TenantKernel:
    tenant_id: int
    adapter_id: int
    backend: str
    artifact: str
    symbol: str
    enabled: bool = True


class StageMLTenantRouter:
    def __init__(self, kernels: dict[int, TenantKernel]):
        self.kernels = dict(kernels)
        self._tables: dict[torch.device, torch.Tensor] = {}

    @classmethod
    def from_manifest(cls, path: str | Path) -> "StageMLTenantRouter":
        """Router over the enabled entries of a kernel manifest (a TenantKernel has the entry's fields)."""
        return cls({e.tenant_id: TenantKernel(**asdict(e)) for e in read_kernel_manifest(path).entries if e.enabled})

    def has_kernel(self, tenant_id: int) -> bool:
        e = self.kernels.get(int(tenant_id))
        return e is not None and e.enabled

    def _table(self, device: torch.device) -> torch.Tensor:
        t = self._tables.get(device)
        if t is None:
            enabled = [tid for tid, k in self.kernels.items() if k.enabled and tid >= 0]
            t = torch.zeros(max(enabled, default=-1) + 2, dtype=torch.bool, device=device)
            if enabled:
                t[torch.tensor(enabled, device=device)] = True
            self._tables[device] = t
        return t

    def materialized_mask(self, tenant_ids: torch.Tensor) -> torch.Tensor:
        """Per-token bool mask of tenants with a kernel, computed where tenant_ids live."""
        table = self._table(tenant_ids.device)
        ids = tenant_ids.reshape(-1).to(torch.long)
        in_range = (ids >= 0) & (ids < table.numel() - 1)
        return table[torch.where(in_range, ids, torch.full_like(ids, table.numel() - 1))] & in_range


# Locations of vLLM's fused_experts across releases, in the order they are tried.
_VLLM_FUSED_EXPERTS_PATHS = ("vllm.model_executor.layers.fused_moe.fused_moe.fused_experts",
                             "vllm.model_executor.layers.fused_moe.fused_experts")


def resolve_vllm_fused_experts() -> tuple[Callable[..., Any] | None, str]:
    """vLLM's fused_experts and its dotted path, or None and why every location failed
    (stageml/vllm_stage_router.py:65-80: same locations, order and messages)."""
    why: list[str] = []
    for path in _VLLM_FUSED_EXPERTS_PATHS:
        module, _, name = path.rpartition(".")
        try:
            fn = getattr(importlib.import_module(module), name)
        except Exception as exc:  # vLLM absent, or this release keeps the function elsewhere
            why.append(f"{path}: {exc}")
            continue
        if callable(fn):
            return fn, path
        why.append(f"{path} exists but is not callable")
    return None, "; ".join(why)


def call_vllm_fused_experts(fn: Callable[..., Any], hidden, gate_up, down, topk_weights, topk_ids):
    """Call vLLM's fused_experts in whichever argument form its release accepts
    (stageml/vllm_stage_router.py:84-105: keywords with inplace=False, then positional with
    inplace=False, then positional; the last failure is reported)."""
    ids = topk_ids.to(dtype=torch.long).contiguous()
    wts = topk_weights.contiguous()
    positional = (hidden, gate_up, down, wts, ids)
    forms = (((), dict(hidden_states=hidden, w1=gate_up, w2=down, topk_weights=wts, topk_ids=ids, inplace=False)),
             (positional + (False,), {}),
             (positional, {}))
    failure: Exception | None = None
    for args, kwargs in forms:
        try:
            return fn(*args, **kwargs)
        except Exception as exc:  # another release's signature (or a failing call): try the next form
            failure = exc
    raise RuntimeError(f"could not call vLLM fused_experts: {failure}")


def call_stageml_residual_op(hidden, gate_up, down, topk_weights, topk_ids):
    if not ensure_stageml_custom_op(allow_python_fallback=True):
        raise RuntimeError("StageML residual custom op is not available")
    return torch.ops.stageml.residual_moe(hidden, gate_up, down, topk_weights, topk_ids)


def route_fused_experts(*, hidden, gate_up, down, topk_weights, topk_ids, tenant_ids, router: StageMLTenantRouter,
                        vllm_fused_experts: Callable[..., Any] | None = None,
                        stageml_op: Callable[..., torch.Tensor] | None = None, split: str = "indexed",
                        weight_sets=None):
    """Route tokens between the StageML residual op and vLLM fused experts (stageml/vllm_stage_router.py:114-157).

    split="indexed" (the reference's behaviour): each backend runs on its own tokens.
    split="masked": no host synchronisation; both backends run on every token with the
    routing weights of the other backend's tokens zeroed, and the outputs are summed.
    A fused-MoE output row is a routing-weighted sum of expert outputs, so a token
    with all-zero weights contributes an exact zero row and each token's row is its
    own backend's row (the same bits when a backend's rows do not depend on the rest
    of its batch, as for this package's op).
    split="device": one ``moe_forward`` call for the whole batch, no host read and no
    vLLM call. Tokens of tenants with an enabled kernel take their rows of
    ``weight_sets.fold_slot`` (tenant id = row; their folded experts run on the folded
    sets, the others on the base experts); all other tokens run on the base experts
    (``weight_sets`` base experts, or ``gate_up`` / ``down`` without weight sets).
    """
    if split not in ("indexed", "masked", "device"):
        raise ValueError(f"split must be 'indexed', 'masked' or 'device', not {split!r}")
    if hidden.shape[0] != tenant_ids.numel():
        raise ValueError("tenant_ids must contain one tenant id per token")
    if split == "device":
        return _route_on_device(hidden, gate_up, down, topk_weights, topk_ids, tenant_ids, router, weight_sets)
    if vllm_fused_experts is None:
        vllm_fused_experts, source = resolve_vllm_fused_experts()
        if vllm_fused_experts is None:
            raise RuntimeError(f"vLLM fused experts could not be resolved: {source}")
    stageml_op = stageml_op or call_stageml_residual_op
    mask = router.materialized_mask(tenant_ids.to(hidden.device))
    if split == "masked":
        m = mask.to(topk_weights.dtype).unsqueeze(1)
        return (stageml_op(hidden, gate_up, down, topk_weights * m, topk_ids)
                + call_vllm_fused_experts(vllm_fused_experts, hidden, gate_up, down, topk_weights * (1 - m), topk_ids))
    n_sel = int(mask.sum())
    if n_sel == hidden.shape[0]:
        return stageml_op(hidden, gate_up, down, topk_weights, topk_ids)
    if n_sel == 0:
        return call_vllm_fused_experts(vllm_fused_experts, hidden, gate_up, down, topk_weights, topk_ids)
    # StageML tokens first, then vLLM's, each in token order: one stable sort, no per-side nonzero.
    order = torch.argsort((~mask).to(torch.uint8), stable=True)
    mine, theirs = order[:n_sel], order[n_sel:]

    def rows(t, idx):
        return t.index_select(0, idx).contiguous()

    out = hidden.new_empty((hidden.shape[0], down.shape[1]))
    out.index_copy_(0, mine, stageml_op(rows(hidden, mine), gate_up, down, rows(topk_weights, mine),
                                        rows(topk_ids, mine)))
    out.index_copy_(0, theirs, call_vllm_fused_experts(vllm_fused_experts, rows(hidden, theirs), gate_up, down,
                                                       rows(topk_weights, theirs), rows(topk_ids, theirs)))
    return out


def _route_on_device(hidden, gate_up, down, topk_weights, topk_ids, tenant_ids, router, weight_sets):
    from . import ops

    ids = topk_ids.contiguous()
    wts = topk_weights.contiguous()
    if weight_sets is None or weight_sets.n_fold == 0:
        gu = gate_up if weight_sets is None else weight_sets.base_gate_up()
        dn = down if weight_sets is None else weight_sets.down
        return ops.moe_forward(hidden.contiguous(), gu, dn, topk_ids=ids, topk_weights=wts)
    mask = router.materialized_mask(tenant_ids.to(hidden.device))
    n = int(weight_sets.fold_slot.shape[0])
    ten = tenant_ids.reshape(-1).to(device=hidden.device, dtype=torch.int32)
    ten = torch.where(mask & (ten >= 0) & (ten < n), ten, torch.full_like(ten, -1))  # table lookups, on the device
    return ops.moe_forward(hidden.contiguous(), weight_sets.gate_up, weight_sets.down, topk_ids=ids,
                           topk_weights=wts, tenant_ids=ten, n_tenants=n, **weight_sets.moe_kwargs())


__all__ = ["KernelManifestEntry", "KernelManifest", "read_kernel_manifest", "write_kernel_manifest", "TenantKernel",
           "StageMLTenantRouter", "resolve_vllm_fused_experts", "call_vllm_fused_experts", "call_stageml_residual_op",
           "route_fused_experts"]
