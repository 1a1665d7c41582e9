"""Synthetic workload generators and stage-0 packing helpers (CPU)."""

import math

import numpy as np
import torch

from stageml_b200 import _packing
from stageml_b200.workloads import MOE_CONFIGS, MoEConfig, make_moe_workload, make_single_lora


def test_mixtral_config_flops_match_the_roofline_table():
    fl = MOE_CONFIGS["mixtral_moe_lora"].flops()
    assert abs(fl["base"] - 1.443e12) / 1.443e12 < 1e-3
    assert abs(fl["total"] - 1.450e12) / 1.450e12 < 2e-3


def test_small_moe_workload_shapes_and_distributions():
    cfg = MoEConfig("t", T=64, H=64, I=96, E=4, k=2, n_shared=1, n_tenants=5, rank=16, tenant_dist="zipf")
    w = make_moe_workload(cfg, device="cpu", seed=0)
    assert w["gate_up"].shape == (5, 192, 64) and w["down"].shape == (5, 64, 96)
    assert w["lora_a13"].shape == (5, 5, 32, 64) and w["lora_b2"].shape == (5, 5, 64, 16)
    assert w["router_w"].shape == (4, 64) and w["router_w"].dtype == torch.float32
    assert abs(w["gate_up"].float().std().item() - 1 / math.sqrt(64)) < 0.01
    assert int(w["tenant_ids"].min()) >= 0 and int(w["tenant_ids"].max()) < 5
    w2 = make_moe_workload(cfg, device="cpu", seed=0)
    assert torch.equal(w["x"], w2["x"]) and torch.equal(w["lora_b13"], w2["lora_b13"])


def test_single_lora_config():
    w = make_single_lora(device="cpu", dim=64, rank=16)
    assert w["scale"] == 2.0 and w["W"].shape == (64, 64) and w["A"].shape == (64, 16)


def test_padding_helpers_are_exact():
    assert _packing.padded_rank(2) == 8 and _packing.padded_rank(8) == 8 and _packing.padded_rank(9) == 16
    assert _packing.padded_rank(17) == 32 and _packing.padded_rank(0) == 0
    A = [torch.randn(3, 10, 6), torch.randn(3, 2, 6)]
    B = [torch.randn(3, 5, 10), torch.randn(3, 5, 2)]
    a, b = _packing.pack_lora_bank([x.transpose(1, 2) for x in [torch.randn(3, 6, 10)]] * 0 + [A[0].transpose(1, 2)
                                   .transpose(1, 2), A[1]], B, 8, 8, 16, torch.float32, "cpu")
    assert a.shape == (2, 3, 16, 8) and b.shape == (2, 3, 8, 16)
    x = torch.randn(7, 6)
    for i in range(2):
        ref = (x @ A[i][0].t()) @ B[i][0].t()
        got = (_packing.pad_last(x, 8) @ a[i, 0].t()) @ b[i, 0].t()
        np.testing.assert_allclose(got[:, :5].numpy(), ref.numpy(), rtol=1e-5, atol=1e-5)
