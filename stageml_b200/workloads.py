"""Seeded synthetic workloads of the five residual-path configurations.

The reference measures on real Mixtral / Qwen checkpoints and PEFT adapters
that are not available here; these generators produce inputs with the same
shapes, dtypes and value distributions (weights N(0, 1/fan_in), activations
N(0, 1), LoRA A ~ N(0, 1/in), B ~ N(0, 1/rank)). Per-token tenant ids follow
the reference's request sampler ``sample_tenants``
(benchmarks/multitenant_bta_system_bench.py:80-101): ``random.Random(seed)``
with ``randrange`` (uniform) or ``choices`` over Zipf weights 1/(i+1)^alpha.

Large tensors can be generated directly on the GPU (``gen_device="cuda"``) so
a multi-GB workload is ready in seconds; parity tests generate on the CPU.
"""

from __future__ import annotations

import math
import random
from dataclasses import dataclass, field

import torch

DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def zipf_probs(n: int, alpha: float) -> list[float]:
    w = [1.0 / ((i + 1) ** alpha) for i in range(n)]
    s = sum(w)
    return [x / s for x in w]


def sample_tenants(n: int, tenants: int, distribution: str, alpha: float = 1.1, burst: int = 1,
                   seed: int = 0) -> list[int]:
    """Per-request tenant ids, same sampler as the reference benchmark."""
    rng = random.Random(seed)
    if distribution == "uniform":
        return [rng.randrange(tenants) for _ in range(n)]
    if distribution == "zipf":
        return rng.choices(list(range(tenants)), weights=zipf_probs(tenants, alpha), k=n)
    if distribution == "round_robin":
        return [i % tenants for i in range(n)]
    if distribution == "bursty":
        out: list[int] = []
        probs = zipf_probs(tenants, alpha)
        while len(out) < n:
            t = rng.choices(list(range(tenants)), weights=probs, k=1)[0]
            out.extend([t] * max(1, burst))
        return out[:n]
    raise ValueError(f"unknown tenant distribution {distribution}")


class _Gen:
    """Seeded normal sampler on a chosen device; outputs cast to the target device/dtype."""

    def __init__(self, seed: int, gen_device: str, device):
        self.g = torch.Generator(device=gen_device)
        self.g.manual_seed(seed)
        self.gen_device = gen_device
        self.device = torch.device(device)

    def normal(self, shape, std: float, dtype: torch.dtype) -> torch.Tensor:
        t = torch.randn(*shape, generator=self.g, device=self.gen_device, dtype=torch.float32)
        if std != 1.0:
            t.mul_(std)
        return t.to(device=self.device, dtype=dtype)

    def normal_stacked(self, n: int, shape, std: float, dtype: torch.dtype) -> torch.Tensor:
        """n independent draws of `shape`, generated one slice at a time (bounded fp32 temporaries)."""
        out = torch.empty((n, *shape), device=self.device, dtype=dtype)
        for i in range(n):
            out[i] = self.normal(shape, std, dtype)
        return out


# ------------------------------------------------------------------ MoE configs
@dataclass
class MoEConfig:
    name: str
    T: int
    H: int
    I: int
    E: int
    k: int
    n_shared: int
    n_tenants: int
    rank: int
    tenant_dist: str
    alpha: float = 1.1
    act_dtype: str = "bf16"
    weight_dtype: str = "bf16"   # or "e4m3"
    lora_scale: float = 2.0
    lora_on: tuple = ("w1", "w3", "w2")

    @property
    def E_tot(self) -> int:
        return self.E + self.n_shared

    @property
    def bank_rank(self) -> int:
        """Rank of the LoRA banks as stored: the adapter rank zero-padded to 8, 16 or 32."""
        from ._packing import padded_rank

        return padded_rank(self.rank)

    def flops(self, T: int | None = None) -> dict:
        """Algorithmic FLOPs (2 x MACs) of one layer call."""
        T = self.T if T is None else T
        P = T * (self.k + self.n_shared)
        base = 2.0 * P * (2 * self.I * self.H + self.H * self.I)
        r = self.rank
        lora = 0.0
        if "w1" in self.lora_on or "w3" in self.lora_on:
            lora += 2.0 * P * (2 * r * self.H + 2 * self.I * r)
        if "w2" in self.lora_on:
            lora += 2.0 * P * (r * self.I + self.H * r)
        router = 2.0 * T * self.H * self.E
        gate_up = 2.0 * P * 2 * self.I * self.H
        return {"base": base, "lora": lora, "router": router, "total": base + lora + router, "gate_up": gate_up}


MOE_CONFIGS = {
    "mixtral_moe_lora": MoEConfig("mixtral_moe_lora", T=2048, H=4096, I=14336, E=8, k=2, n_shared=0, n_tenants=32,
                                  rank=16, tenant_dist="uniform"),
    "fine_grained_fp8_moe_lora": MoEConfig("fine_grained_fp8_moe_lora", T=8192, H=2048, I=1408, E=64, k=6,
                                           n_shared=2, n_tenants=128, rank=8, tenant_dist="zipf",
                                           weight_dtype="e4m3"),
}


def make_moe_workload(cfg: MoEConfig, *, device="cuda", gen_device: str | None = None, seed: int = 0,
                      T: int | None = None) -> dict:
    """Weights, router, LoRA banks and one batch of tokens for a MoE-LoRA config.

    Returned layouts follow the C ABI: gate_up [E_tot, 2I, H] (rows [:I] = w1,
    the SiLU branch), down [E_tot, H, I], router_w [E, H] fp32 (= W_g^T),
    lora_a13 [n_tenants, E_tot, 2r, H], lora_b13 [n_tenants, E_tot, 2I, r],
    lora_a2 [n_tenants, E_tot, r, I], lora_b2 [n_tenants, E_tot, H, r], with
    r = cfg.bank_rank: factors of rank cfg.rank are drawn, then zero-padded
    (rows of A, columns of B), which leaves every product unchanged.
    """
    gen_device = gen_device or ("cuda" if torch.device(device).type == "cuda" else "cpu")
    T = cfg.T if T is None else T
    g = _Gen(seed, gen_device, device)
    act = DTYPES[cfg.act_dtype]
    H, I, E, Et, r, nT = cfg.H, cfg.I, cfg.E, cfg.E_tot, cfg.rank, cfg.n_tenants
    w = {}
    w["x"] = g.normal((T, H), 1.0, act)
    w["router_w"] = g.normal((H, E), 1.0 / math.sqrt(H), torch.float32).t().contiguous()
    w["gate_up"] = g.normal_stacked(Et, (2 * I, H), 1.0 / math.sqrt(H), act)
    w["down"] = g.normal_stacked(Et, (H, I), 1.0 / math.sqrt(I), act)
    if r == 0:  # no adapters
        w["lora_a13"] = w["lora_b13"] = w["lora_a2"] = w["lora_b2"] = None
    else:
        a13 = g.normal_stacked(nT * Et, (2 * r, H), 1.0 / math.sqrt(H), act).view(nT, Et, 2 * r, H)
        b13 = g.normal_stacked(nT * Et, (2 * I, r), 1.0 / math.sqrt(r), act).view(nT, Et, 2 * I, r)
        a2 = g.normal_stacked(nT * Et, (r, I), 1.0 / math.sqrt(I), act).view(nT, Et, r, I)
        b2 = g.normal_stacked(nT * Et, (H, r), 1.0 / math.sqrt(r), act).view(nT, Et, H, r)
        rp = cfg.bank_rank
        if rp != r:
            pad = lambda t, dim: torch.cat([t, t.new_zeros(t.shape[:dim] + (rp - r,) + t.shape[dim + 1:])], dim)
            a13 = torch.cat([pad(a13[:, :, :r], 2), pad(a13[:, :, r:], 2)], 2).contiguous()
            b13 = pad(b13, 3).contiguous()
            a2 = pad(a2, 2).contiguous()
            b2 = pad(b2, 3).contiguous()
            r = rp
        if "w1" not in cfg.lora_on:
            a13[:, :, :r].zero_()
        if "w3" not in cfg.lora_on:
            a13[:, :, r:].zero_()
        w["lora_a13"], w["lora_b13"] = a13, b13
        w["lora_a2"], w["lora_b2"] = (a2, b2) if "w2" in cfg.lora_on else (None, None)
    w["lora_scale"] = torch.full((nT,), cfg.lora_scale, dtype=torch.float32, device=device)
    ten = sample_tenants(T, nT, cfg.tenant_dist, cfg.alpha, seed=seed)
    w["tenant_ids"] = torch.tensor(ten, dtype=torch.int32, device=device)
    w["gate_up_scale"] = w["down_scale"] = None
    if cfg.weight_dtype == "e4m3":
        from . import ops

        w["gate_up"], w["gate_up_scale"] = ops.quantize_e4m3_rows(w["gate_up"])
        w["down"], w["down_scale"] = ops.quantize_e4m3_rows(w["down"])
    return w


def moe_bytes(cfg: MoEConfig, w: dict, T: int | None = None) -> dict:
    """Algorithmic bytes of one layer call: unique weights + touched adapter slices + activations in/out."""
    T = cfg.T if T is None else T
    esz = 1 if cfg.weight_dtype == "e4m3" else 2
    weights = cfg.E_tot * 3 * cfg.H * cfg.I * esz
    if cfg.weight_dtype == "e4m3":
        weights += cfg.E_tot * (2 * cfg.I + cfg.H) * 4
    acts = 2 * T * cfg.H * 2
    per_pair_adapter = 2 * (2 * cfg.rank * cfg.H + 2 * cfg.I * cfg.rank + cfg.rank * cfg.I + cfg.H * cfg.rank)
    return {"weights": weights, "activations": acts, "adapter_per_pair": per_pair_adapter}


# ------------------------------------------------------------ dense configs
def make_single_lora(seed: int = 0, device="cuda", gen_device: str | None = None, M: int = 1, dim: int = 4096,
                     rank: int = 16, alpha: float = 32.0) -> dict:
    """Config 1: fp32 x[1,4096], W[4096,4096] ([in,out]), A[4096,16], B[16,4096], scale alpha/rank = 2."""
    gen_device = gen_device or ("cuda" if torch.device(device).type == "cuda" else "cpu")
    g = _Gen(seed, gen_device, device)
    return {
        "x": g.normal((M, dim), 1.0, torch.float32),
        "W": g.normal((dim, dim), 1.0 / math.sqrt(dim), torch.float32),
        "A": g.normal((dim, rank), 1.0 / math.sqrt(dim), torch.float32),
        "B": g.normal((rank, dim), 1.0 / math.sqrt(rank), torch.float32),
        "scale": alpha / rank,
    }


def make_adapter_bank(seed: int = 0, device="cuda", gen_device: str | None = None, M: int = 256, dim: int = 4096,
                      n_adapters: int = 64, rank: int = 16, n_folded: int = 8, alpha_zipf: float = 1.1,
                      dtype: str = "bf16") -> dict:
    """Config 2: x[256,4096], W[4096,4096], 64 rank-16 adapters (scale 2), Zipf(1.1) ids, top-8 folded."""
    gen_device = gen_device or ("cuda" if torch.device(device).type == "cuda" else "cpu")
    g = _Gen(seed, gen_device, device)
    dt = DTYPES[dtype]
    ids = sample_tenants(M, n_adapters, "zipf", alpha_zipf, seed=seed)
    counts = {}
    for a in ids:
        counts[a] = counts.get(a, 0) + 1
    folded = sorted(counts, key=lambda a: (-counts[a], f"adapter_{a}"))[:n_folded]
    return {
        "x": g.normal((M, dim), 1.0, dt),
        "W": g.normal((dim, dim), 1.0 / math.sqrt(dim), dt),
        "A": g.normal((n_adapters, rank, dim), 1.0 / math.sqrt(dim), dt),
        "B": g.normal((n_adapters, dim, rank), 1.0 / math.sqrt(rank), dt),
        "scale": 2.0,
        "adapter_ids": ids,
        "folded": folded,
    }


LLAMA_PROJ = {"q": (4096, 4096), "k": (4096, 4096), "v": (4096, 4096), "o": (4096, 4096), "gate": (11008, 4096),
              "up": (11008, 4096), "down": (4096, 11008)}


def make_llama_block(seed: int = 0, device="cuda", gen_device: str | None = None, batch: int = 16, seq: int = 128,
                     n_tenants: int = 16, rank: int = 16, dtype: str = "fp16", scale: float = 2.0) -> dict:
    """Config 3: LLaMA-7B block projections with rank-16 LoRA on all 7, one tenant per sequence."""
    gen_device = gen_device or ("cuda" if torch.device(device).type == "cuda" else "cpu")
    g = _Gen(seed, gen_device, device)
    dt = DTYPES[dtype]
    M = batch * seq
    rng = random.Random(seed)
    seq_tenant = [rng.randrange(n_tenants) for _ in range(batch)]
    row_tenant = torch.tensor([t for t in seq_tenant for _ in range(seq)], dtype=torch.int32, device=device)
    out = {"x": g.normal((M, 4096), 1.0, dt), "x_o": g.normal((M, 4096), 1.0, dt), "row_tenant": row_tenant,
           "scale": scale, "proj": {}}
    for name, (n_out, n_in) in LLAMA_PROJ.items():
        out["proj"][name] = {
            "W": g.normal((n_out, n_in), 1.0 / math.sqrt(n_in), dt),
            "A": g.normal((n_tenants, rank, n_in), 1.0 / math.sqrt(n_in), dt),
            "B": g.normal((n_tenants, n_out, rank), 1.0 / math.sqrt(rank), dt),
        }
    return out


__all__ = ["zipf_probs", "sample_tenants", "MoEConfig", "MOE_CONFIGS", "make_moe_workload", "moe_bytes",
           "make_single_lora", "make_adapter_bank", "make_llama_block", "LLAMA_PROJ", "DTYPES"]
