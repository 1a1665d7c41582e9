"""The Mixtral-shape MoE-LoRA layer at its full benchmark size (T=2048, H=4096,
I=14336, E=8, top-2, rank-16 LoRA on w1/w3/w2, 32 tenants): size-independent
properties, an oracle check on the tokens routed to the most common expert pair,
and one on sampled tokens over every expert (tile pairs and odd trailing tiles)."""

import numpy as np
import pytest
import torch

from conftest import oracle_moe_tokens, rel_l2
from oracle import moe as omoe

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def layer():
    import stageml_b200.ops as ops
    from stageml_b200.workloads import MOE_CONFIGS, make_moe_workload

    cfg = MOE_CONFIGS["mixtral_moe_lora"]
    w = make_moe_workload(cfg, device=DEV, seed=0)

    def call(x, ten, **over):
        kw = dict(router_w=w["router_w"], k=cfg.k, tenant_ids=ten, n_tenants=cfg.n_tenants, rank=cfg.bank_rank,
                  lora_a13=w["lora_a13"], lora_b13=w["lora_b13"], lora_a2=w["lora_a2"], lora_b2=w["lora_b2"],
                  lora_scale=w["lora_scale"])
        kw.update(over)
        return ops.moe_forward(x, w["gate_up"], w["down"], **kw)

    return cfg, w, call, ops


def test_full_size_deterministic_and_order_invariant(layer):
    cfg, w, call, ops = layer
    y1 = call(w["x"], w["tenant_ids"])
    y2 = call(w["x"], w["tenant_ids"])
    assert torch.equal(y1, y2)
    perm = torch.randperm(cfg.T, generator=torch.Generator().manual_seed(3)).to(DEV)
    y3 = call(w["x"][perm].contiguous(), w["tenant_ids"][perm].contiguous())
    assert torch.equal(y3, y1[perm])
    assert ops.take_status(y1) == 0
    assert torch.isfinite(y1.float()).all()


def test_full_size_against_oracle_on_two_experts(layer):
    cfg, w, call, ops = layer
    y = call(w["x"], w["tenant_ids"])
    ids, wts, _ = ops.route_topk(w["x"], w["router_w"], cfg.k, True)
    ids = ids.cpu().numpy()
    pairs, counts = np.unique(np.sort(ids, 1), axis=0, return_counts=True)
    e0, e1 = pairs[np.argmax(counts)]
    sel = np.nonzero(np.all(np.isin(ids, [e0, e1]), 1))[0][:48]
    assert sel.size >= 8
    f32 = lambda t: t.float().cpu().numpy()
    ex = [int(e0), int(e1)]
    remap = np.where(ids[sel] == e0, 0, 1)
    ref = omoe.moe_forward(f32(w["x"][sel]), f32(w["gate_up"][ex]), f32(w["down"][ex]), remap, wts.cpu().numpy()[sel],
                           tenant_ids=w["tenant_ids"].cpu().numpy()[sel], lora_a13=f32(w["lora_a13"][:, ex]),
                           lora_b13=f32(w["lora_b13"][:, ex]), lora_a2=f32(w["lora_a2"][:, ex]),
                           lora_b2=f32(w["lora_b2"][:, ex]), lora_scale=f32(w["lora_scale"]), dtype=np.float64)
    assert rel_l2(y.float().cpu().numpy()[sel], ref) < 1e-2


def test_full_size_batch_of_one(layer):
    """Decode-sized batches (at most 16 routed rows) take the weight-streaming GEMM,
    larger ones the tensor-memory GEMM. Within each path a token's output does not
    depend on the rest of the batch (bit-identical); across the two paths the sums
    run in different orders and agree within the bf16 tolerance (rel-L2 <= 1e-2)."""
    cfg, w, call, ops = layer
    x, ten = w["x"], w["tenant_ids"]
    y1 = call(x[:1].contiguous(), ten[:1].contiguous())
    y8 = call(x[:8].contiguous(), ten[:8].contiguous())
    y64 = call(x[:64].contiguous(), ten[:64].contiguous())
    y128 = call(x[:128].contiguous(), ten[:128].contiguous())
    assert torch.equal(y1[0], y8[0])
    assert torch.equal(y64, y128[:64])
    assert rel_l2(y8.float().cpu().numpy(), y64[:8].float().cpu().numpy()) < 1e-2
    assert ops.take_status(y1) == 0


def test_full_size_against_oracle_on_every_expert(layer):
    """Tokens of the first and last tenants, checked over every expert they are routed to.

    Rows of an expert's segment are sorted by tenant, so the last tenant's rows sit in
    each expert's trailing tile (the odd tile beside the tile pairs, where an expert has
    an odd tile count) and the first tenant's rows in its leading tile pair."""
    cfg, w, call, ops = layer
    y = call(w["x"], w["tenant_ids"])
    ids, wts, _ = ops.route_topk(w["x"], w["router_w"], cfg.k, True)
    ids, wts = ids.cpu().numpy(), wts.cpu().numpy()
    ten = w["tenant_ids"].cpu().numpy()
    sel = np.concatenate([np.nonzero(ten == 0)[0][:12], np.nonzero(ten == cfg.n_tenants - 1)[0][:20]])
    assert set(np.unique(ids[sel])) == set(range(cfg.E))
    f32 = lambda t: t.float().cpu().numpy()
    xs = f32(w["x"])
    ref = oracle_moe_tokens(np.arange(sel.size), ids[sel], wts[sel], ten[sel], xs[sel],
                            lambda e: (f32(w["gate_up"][e]), f32(w["down"][e])),
                            lambda e: tuple(f32(w[n][:, e:e + 1]) for n in ("lora_a13", "lora_b13", "lora_a2", "lora_b2")),
                            f32(w["lora_scale"]), n_routed=cfg.E)
    assert rel_l2(y.float().cpu().numpy()[sel], ref) < 1e-2
    assert ops.take_status(y) == 0
