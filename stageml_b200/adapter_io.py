"""PEFT expert-LoRA checkpoints -> the MoE layer's adapter banks.

``load_expert_lora_adapter`` reads one adapter the way the reference's real
benchmark does (``load_expert_lora_adapter``, ``_normalize_lora_key``,
``_expert_index_from_name``, ``_load_state_dict``;
benchmarks/real_moe_lora_residual_bench.py:30-46, 65-69, 172-216): keys lose
``.default.`` and ``base_model.model.``; the expert index is the number after
``experts.`` / ``experts_``; only keys of the chosen projection count (``w1`` by
default, or ``$LORA_PROJECTION``); A is a ``lora_A`` matrix ``[r, in]``, B a
``lora_B`` matrix ``[out, r]``; the rank is the most common one among the experts
that have both; experts without a matching pair stay zero; scaling 1.0.

``load_moe_lora_banks`` packs several adapters (w1, w3 and w2 of each) into the
banks ``ops.moe_forward`` takes -- ``lora_a13 [n, E, 2r, H]``, ``lora_b13 [n, E,
2I, r]``, ``lora_a2 [n, E, r, I]``, ``lora_b2 [n, E, H, r]``, ``lora_scale [n]`` --
for all experts or one contiguous shard of them (expert parallel), with the
rank padded to 8, 16 or 32 and the scale lora_alpha / r from the adapter's
``adapter_config.json`` (alpha / sqrt(r) with ``use_rslora``), 1.0 without one.
"""

from __future__ import annotations

import json
import math
import os
import re
from pathlib import Path

import torch

from ._packing import padded_rank
from .moe_lora_layers import MoEAdapterSpec

__all__ = ["load_expert_lora_adapter", "load_moe_lora_banks", "adapter_scaling"]

_EXPERT = re.compile(r"experts[\._](\d+)")


def _load_state_dict(path: Path) -> dict:
    files = sorted(path.glob("*.safetensors")) + sorted(path.glob("*.bin")) + sorted(path.glob("*.pt"))
    if not files:
        raise FileNotFoundError(f"no adapter checkpoint files found in {path}")
    f = files[0]
    if f.suffix == ".safetensors":
        from safetensors.torch import load_file

        return load_file(str(f))
    obj = torch.load(str(f), map_location="cpu", weights_only=True)
    if isinstance(obj, dict) and isinstance(obj.get("state_dict"), dict):
        return obj["state_dict"]
    if not isinstance(obj, dict):
        raise ValueError(f"unsupported checkpoint object in {f}")
    return obj


def _normalize_key(key: str) -> str:
    return key.replace(".default.", ".").replace("base_model.model.", "")


def load_expert_lora_adapter(adapter_dir, *, num_experts: int, in_features: int, out_features: int,
                             projection: str | None = None) -> MoEAdapterSpec:
    """One projection of an expert-LoRA checkpoint as ``MoEAdapterSpec`` (A [E, r, in], B [E, out, r], fp32)."""
    adapter_dir = Path(adapter_dir)
    proj = (projection if projection is not None else os.environ.get("LORA_PROJECTION", "w1")).strip().lower()
    sd = {_normalize_key(k): v for k, v in _load_state_dict(adapter_dir).items() if isinstance(v, torch.Tensor)}
    pairs: dict[int, dict[str, torch.Tensor]] = {e: {} for e in range(num_experts)}
    for key, t in sd.items():
        m = _EXPERT.search(key)
        if m is None or int(m.group(1)) >= num_experts:
            continue
        lk = key.lower()
        if proj and f".{proj}." not in lk:
            continue
        e = int(m.group(1))
        if "lora_a" in lk and t.ndim == 2 and t.shape[1] == in_features:
            pairs[e]["A"] = t.detach().cpu().to(torch.float32)
        if "lora_b" in lk and t.ndim == 2 and t.shape[0] == out_features:
            pairs[e]["B"] = t.detach().cpu().to(torch.float32)
    ranks = [p["A"].shape[0] for p in pairs.values() if "A" in p and "B" in p]
    if not ranks:
        raise RuntimeError(f"could not find expert LoRA A and B tensors in {adapter_dir}")
    rank = max(sorted(set(ranks)), key=ranks.count)  # most common; the smallest of tied ranks
    A = torch.zeros(num_experts, rank, in_features, dtype=torch.float32)
    B = torch.zeros(num_experts, out_features, rank, dtype=torch.float32)
    found = 0
    for e, p in pairs.items():
        if "A" in p and "B" in p and p["A"].shape[0] == rank and p["B"].shape[1] == rank:
            A[e], B[e] = p["A"], p["B"]
            found += 1
    if found == 0:
        raise RuntimeError(f"found adapter tensors in {adapter_dir} but no tensors matched rank and shape")
    return MoEAdapterSpec(name=adapter_dir.name, A=A, B=B, scaling=1.0)


def adapter_scaling(adapter_dir, rank: int) -> float:
    """lora_alpha / r (alpha / sqrt(r) with use_rslora) from adapter_config.json; 1.0 without it."""
    cfg_path = Path(adapter_dir) / "adapter_config.json"
    if not cfg_path.exists():
        return 1.0
    cfg = json.loads(cfg_path.read_text())
    r = int(cfg.get("r", rank) or rank)
    alpha = float(cfg.get("lora_alpha", r))
    return alpha / math.sqrt(r) if cfg.get("use_rslora") else alpha / r


def load_moe_lora_banks(adapter_dirs, *, num_experts: int, hidden: int, intermediate: int,
                        expert_range: tuple[int, int] | None = None, dtype=torch.bfloat16, device="cuda") -> dict:
    """Banks of ``ops.moe_forward`` for the adapters in ``adapter_dirs`` (tenant i = adapter i).

    A projection an adapter does not train stays zero; an adapter with no expert LoRA at
    all is an error. ``expert_range`` = (first, end) packs only those experts (a shard).
    """
    e0, e1 = expert_range if expert_range is not None else (0, num_experts)
    if not 0 <= e0 < e1 <= num_experts:
        raise ValueError(f"expert range {expert_range} outside [0, {num_experts})")
    H, I = hidden, intermediate
    shapes = {"w1": (H, I), "w3": (H, I), "w2": (I, H)}
    specs = []
    for d in adapter_dirs:
        got = {}
        for proj, (din, dout) in shapes.items():
            try:
                got[proj] = load_expert_lora_adapter(d, num_experts=num_experts, in_features=din, out_features=dout,
                                                     projection=proj)
            except RuntimeError:
                got[proj] = None
        if all(v is None for v in got.values()):
            raise RuntimeError(f"no expert LoRA of w1, w3 or w2 in {d}")
        specs.append(got)
    r = max(s.rank for got in specs for s in got.values() if s is not None)
    rp = padded_rank(r)
    n, E = len(specs), e1 - e0
    a13 = torch.zeros((n, E, 2 * rp, H), dtype=dtype, device=device)
    b13 = torch.zeros((n, E, 2 * I, rp), dtype=dtype, device=device)
    a2 = torch.zeros((n, E, rp, I), dtype=dtype, device=device)
    b2 = torch.zeros((n, E, H, rp), dtype=dtype, device=device)
    scale = torch.ones(n, dtype=torch.float32)
    to = lambda t: t[e0:e1].to(device=device, dtype=dtype)
    for t, (d, got) in enumerate(zip(adapter_dirs, specs)):
        w1, w3, w2 = got["w1"], got["w3"], got["w2"]
        if w1 is not None:
            a13[t, :, : w1.rank] = to(w1.A)
            b13[t, :, :I, : w1.rank] = to(w1.B)
        if w3 is not None:
            a13[t, :, rp: rp + w3.rank] = to(w3.A)
            b13[t, :, I:, : w3.rank] = to(w3.B)
        if w2 is not None:
            a2[t, :, : w2.rank] = to(w2.A)
            b2[t, :, :, : w2.rank] = to(w2.B)
        scale[t] = adapter_scaling(d, max(s.rank for s in got.values() if s is not None))
    return {"lora_a13": a13, "lora_b13": b13, "lora_a2": a2, "lora_b2": b2,
            "lora_scale": scale.to(device), "rank": rp}
