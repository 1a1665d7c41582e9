"""PEFT expert-LoRA checkpoint loading and bank packing (CPU).

The loader is checked against the reference's own load_expert_lora_adapter on
the same checkpoint (tests/golden/expert_lora_adapter.npz holds the state dict
and the reference's A / B for w1, w3 and w2)."""

import json

import numpy as np
import pytest
import torch

from conftest import load_golden


def _write_checkpoint(tmp_path, fmt="safetensors"):
    g = load_golden("expert_lora_adapter")
    sd = {str(k): torch.from_numpy(g[f"t{i}"]) for i, k in enumerate(g["keys"])}
    if fmt == "safetensors":
        from safetensors.torch import save_file

        save_file(sd, str(tmp_path / "adapter_model.safetensors"))
    else:
        torch.save({"state_dict": sd}, str(tmp_path / "adapter_model.bin"))
    return g, int(g["E"]), int(g["H"]), int(g["I"])


@pytest.mark.parametrize("fmt", ["safetensors", "bin"])
def test_loader_matches_reference(tmp_path, fmt):
    from stageml_b200.adapter_io import load_expert_lora_adapter

    g, E, H, I = _write_checkpoint(tmp_path, fmt)
    for proj, (din, dout) in (("w1", (H, I)), ("w3", (H, I)), ("w2", (I, H))):
        spec = load_expert_lora_adapter(tmp_path, num_experts=E, in_features=din, out_features=dout, projection=proj)
        np.testing.assert_array_equal(spec.A.numpy(), g[f"{proj}_A"], err_msg=proj)
        np.testing.assert_array_equal(spec.B.numpy(), g[f"{proj}_B"], err_msg=proj)
        assert spec.scaling == float(g[f"{proj}_scaling"])


def test_loader_env_projection_and_errors(tmp_path, monkeypatch):
    from stageml_b200.adapter_io import load_expert_lora_adapter

    g, E, H, I = _write_checkpoint(tmp_path)
    monkeypatch.setenv("LORA_PROJECTION", "w2")
    spec = load_expert_lora_adapter(tmp_path, num_experts=E, in_features=I, out_features=H)
    np.testing.assert_array_equal(spec.A.numpy(), g["w2_A"])
    with pytest.raises(RuntimeError):  # no w2 pair has these shapes
        load_expert_lora_adapter(tmp_path, num_experts=E, in_features=H, out_features=I)
    with pytest.raises(FileNotFoundError):
        load_expert_lora_adapter(tmp_path / "missing", num_experts=E, in_features=H, out_features=I)


def test_banks_layout_scale_and_shard(tmp_path):
    from stageml_b200.adapter_io import load_moe_lora_banks

    d0, d1 = tmp_path / "a0", tmp_path / "a1"
    d0.mkdir()
    d1.mkdir()
    g, E, H, I = _write_checkpoint(d0)
    _write_checkpoint(d1)
    (d1 / "adapter_config.json").write_text(json.dumps({"r": 4, "lora_alpha": 8}))
    b = load_moe_lora_banks([d0, d1], num_experts=E, hidden=H, intermediate=I, dtype=torch.float32, device="cpu")
    assert b["rank"] == 8
    assert b["lora_a13"].shape == (2, E, 16, H) and b["lora_b13"].shape == (2, E, 2 * I, 8)
    assert b["lora_a2"].shape == (2, E, 8, I) and b["lora_b2"].shape == (2, E, H, 8)
    assert b["lora_scale"].tolist() == [1.0, 2.0]
    A1, B1, A3, B3 = (torch.from_numpy(g[n]) for n in ("w1_A", "w1_B", "w3_A", "w3_B"))
    assert torch.equal(b["lora_a13"][1, :, :4], A1) and torch.equal(b["lora_a13"][1, :, 8:12], A3)
    assert not b["lora_a13"][:, :, 4:8].any() and not b["lora_a13"][:, :, 12:].any()
    assert torch.equal(b["lora_b13"][0, :, :I, :4], B1) and torch.equal(b["lora_b13"][0, :, I:, :4], B3)
    assert torch.equal(b["lora_a2"][0, :, :4], torch.from_numpy(g["w2_A"]))
    assert torch.equal(b["lora_b2"][0, :, :, :4], torch.from_numpy(g["w2_B"]))
    shard = load_moe_lora_banks([d0], num_experts=E, hidden=H, intermediate=I, expert_range=(1, 3),
                                dtype=torch.float32, device="cpu")
    assert torch.equal(shard["lora_a13"][0], b["lora_a13"][0, 1:3])
    with pytest.raises(ValueError):
        load_moe_lora_banks([d0], num_experts=E, hidden=H, intermediate=I, expert_range=(3, 9), device="cpu")


@pytest.mark.gpu
def test_loaded_banks_drive_the_moe_layer(tmp_path):
    """Banks loaded from a PEFT checkpoint run the CUDA MoE layer; the oracle agrees."""
    from conftest import rel_l2
    from oracle import moe as omoe
    from stageml_b200 import ops
    from stageml_b200.adapter_io import load_moe_lora_banks

    d0, d1 = tmp_path / "a0", tmp_path / "a1"
    d0.mkdir()
    d1.mkdir()
    g, E, H, I = _write_checkpoint(d0)
    _write_checkpoint(d1)
    (d1 / "adapter_config.json").write_text(json.dumps({"r": 4, "lora_alpha": 8}))
    b = load_moe_lora_banks([d0, d1], num_experts=E, hidden=H, intermediate=I, dtype=torch.bfloat16, device="cuda")
    gen = torch.Generator().manual_seed(3)
    T, k = 200, 2
    x = torch.randn(T, H, generator=gen).cuda().to(torch.bfloat16)
    gu = (torch.randn(E, 2 * I, H, generator=gen) * H ** -0.5).cuda().to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=gen) * I ** -0.5).cuda().to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(T)]).cuda()
    w = torch.softmax(torch.randn(T, k, generator=gen), -1).cuda()
    ten = torch.randint(-1, 2, (T,), generator=gen, dtype=torch.int32).cuda()
    y = ops.moe_forward(x, gu, dn, topk_ids=ids, topk_weights=w, tenant_ids=ten, n_tenants=2, rank=b["rank"],
                        lora_a13=b["lora_a13"], lora_b13=b["lora_b13"], lora_a2=b["lora_a2"], lora_b2=b["lora_b2"],
                        lora_scale=b["lora_scale"])
    f = lambda t: t.float().cpu().numpy().astype(np.float64)
    ref = omoe.moe_forward(f(x), f(gu), f(dn), ids.cpu().numpy(), w.cpu().numpy(), tenant_ids=ten.cpu().numpy(),
                           lora_a13=f(b["lora_a13"]), lora_b13=f(b["lora_b13"]), lora_a2=f(b["lora_a2"]),
                           lora_b2=f(b["lora_b2"]), lora_scale=f(b["lora_scale"]))
    assert rel_l2(f(y), ref) < 1e-2
