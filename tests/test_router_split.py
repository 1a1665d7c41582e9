"""Tenant split of the vLLM interception point, with fake backends (as the reference's
tests/test_vllm_stage_router.py), plus the golden split produced by the reference."""

import json

import numpy as np
import pytest
import torch

from conftest import load_golden
from stageml_b200.vllm_stage_router import (KernelManifest, KernelManifestEntry, StageMLTenantRouter, TenantKernel,
                                            route_fused_experts, write_kernel_manifest)


def fake_vllm(hidden, gate_up, down, topk_weights, topk_ids):
    return torch.zeros((hidden.shape[0], down.shape[1]), dtype=hidden.dtype) + 1


def fake_stage(hidden, gate_up, down, topk_weights, topk_ids):
    return torch.zeros((hidden.shape[0], down.shape[1]), dtype=hidden.dtype) + 2


def _call(tenant_ids, router, hidden=None):
    hidden = torch.randn(4, 3) if hidden is None else hidden
    return route_fused_experts(hidden=hidden, gate_up=torch.randn(2, 4, 3), down=torch.randn(2, 3, 2),
                               topk_weights=torch.ones(hidden.shape[0], 1),
                               topk_ids=torch.zeros(hidden.shape[0], 1, dtype=torch.long), tenant_ids=tenant_ids,
                               router=router, vllm_fused_experts=fake_vllm, stageml_op=fake_stage)


def test_router_splits_materialized_and_dynamic_tokens():
    router = StageMLTenantRouter({0: TenantKernel(tenant_id=0, adapter_id=0, backend="t", artifact="x", symbol="s")})
    out = _call(torch.tensor([0, 1, 0, 1]), router)
    assert out.shape == (4, 3)
    assert torch.equal(out[:, 0], torch.tensor([2.0, 1.0, 2.0, 1.0]))


def test_all_and_none_materialized():
    router = StageMLTenantRouter({0: TenantKernel(0, 0, "t", "x", "s")})
    assert torch.equal(_call(torch.tensor([0, 0, 0, 0]), router), torch.full((4, 3), 2.0))
    assert torch.equal(_call(torch.tensor([5, 7, 1, -1]), router), torch.full((4, 3), 1.0))


def test_router_rejects_bad_tenant_shape():
    with pytest.raises(ValueError, match="one tenant id per token"):
        _call(torch.tensor([0, 1]), StageMLTenantRouter({}))


def test_disabled_entries_and_manifest(tmp_path):
    m = KernelManifest(1, "m", (KernelManifestEntry(0, 0, "b", "a"), KernelManifestEntry(2, 1, "b", "a", enabled=False)))
    p = write_kernel_manifest(tmp_path / "k.json", m)
    router = StageMLTenantRouter.from_manifest(p)
    assert router.has_kernel(0) and not router.has_kernel(2) and not router.has_kernel(9)
    assert json.loads(p.read_text())["entries"][1]["enabled"] is False
    np.testing.assert_array_equal(router.materialized_mask(torch.tensor([0, 2, 9, -3])).numpy(),
                                  [True, False, False, False])


def test_golden_split_from_reference():
    g = load_golden("router_split")
    kernels = {int(t): TenantKernel(int(t), 0, "t", "x", "s") for t in g["materialized"]}
    fv = lambda h, gu, dn, *a: torch.zeros((h.shape[0], dn.shape[1])) + 1 + h[:, :1]
    fs = lambda h, gu, dn, *a: torch.zeros((h.shape[0], dn.shape[1])) + 2 + h[:, :1]
    out = route_fused_experts(hidden=torch.from_numpy(g["hidden"]), gate_up=torch.randn(2, 4, 3),
                              down=torch.randn(2, 3, 2), topk_weights=torch.ones(6, 1),
                              topk_ids=torch.zeros(6, 1, dtype=torch.long),
                              tenant_ids=torch.from_numpy(g["tenant_ids"]), router=StageMLTenantRouter(kernels),
                              vllm_fused_experts=fv, stageml_op=fs)
    np.testing.assert_array_equal(out.numpy(), g["out"])


def test_masked_split_needs_no_host_sync_and_matches_indexed():
    """split="masked" runs both backends on every token with the other side's routing
    weights zeroed; for weight-linear backends each row equals the indexed split's."""
    g = torch.Generator().manual_seed(3)
    hidden = torch.randn(7, 3, generator=g)
    w = torch.rand(7, 2, generator=g)
    ids = torch.zeros(7, 2, dtype=torch.long)
    fv = lambda h, gu, dn, tw, ti: (h[:, : dn.shape[1]] * 3.0) * tw.sum(1, keepdim=True)
    fs = lambda h, gu, dn, tw, ti: (h[:, : dn.shape[1]] - 1.0) * tw.sum(1, keepdim=True)
    router = StageMLTenantRouter({0: TenantKernel(0, 0, "t", "x", "s"), 4: TenantKernel(4, 1, "t", "x", "s")})
    ten = torch.tensor([0, 1, 4, 4, -1, 9, 0])
    kw = dict(hidden=hidden, gate_up=torch.randn(2, 4, 3), down=torch.randn(2, 3, 2), topk_weights=w, topk_ids=ids,
              tenant_ids=ten, router=router, vllm_fused_experts=fv, stageml_op=fs)
    a = route_fused_experts(**kw)
    b = route_fused_experts(split="masked", **kw)
    torch.testing.assert_close(b, a, rtol=0, atol=0)
    with pytest.raises(ValueError, match="split"):
        route_fused_experts(split="bogus", **kw)
