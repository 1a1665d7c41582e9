"""Stage-0 packing of weights and adapter factors for the sm_100a kernels.

The kernels want 16-byte row pitches (feature sizes that are multiples of 8)
and LoRA ranks of 8, 16 or 32 (one or two K=16 tensor-core steps; rank 8 fills
the other half of its step with zeros in shared memory). Zero padding
gives identical results: padded input columns meet zero weight columns, padded
output rows are sliced away, and padded rank columns of A / B multiply zeros.
"""

from __future__ import annotations

from typing import Sequence

import torch


def round_up(n: int, m: int) -> int:
    return (n + m - 1) // m * m


def padded_rank(r: int) -> int:
    if r <= 0:
        return 0
    if r <= 8:
        return 8
    if r <= 16:
        return 16
    if r <= 32:
        return 32
    raise ValueError(f"LoRA rank {r} > 32 is not supported by the sm_100a path")


def pad_last(t: torch.Tensor, n: int) -> torch.Tensor:
    if t.shape[-1] == n:
        return t
    out = t.new_zeros((*t.shape[:-1], n))
    out[..., : t.shape[-1]] = t
    return out


def pad_dim(t: torch.Tensor, dim: int, n: int) -> torch.Tensor:
    if t.shape[dim] == n:
        return t
    shape = list(t.shape)
    shape[dim] = n
    out = t.new_zeros(shape)
    idx = [slice(None)] * t.dim()
    idx[dim] = slice(0, t.shape[dim])
    out[tuple(idx)] = t
    return out


def pack_lora_bank(As: Sequence[torch.Tensor], Bs: Sequence[torch.Tensor], k_pad: int, n_pad: int, r_pad: int,
                   dtype: torch.dtype, device) -> tuple[torch.Tensor, torch.Tensor]:
    """Stack per-adapter A [..., r, K] and B [..., N, r] into zero-padded banks
    A [n, ..., r_pad, k_pad] and B [n, ..., n_pad, r_pad]."""
    a_bank, b_bank = [], []
    for A, B in zip(As, Bs):
        A = A.detach().to(device=device, dtype=dtype)
        B = B.detach().to(device=device, dtype=dtype)
        a_bank.append(pad_dim(pad_last(A, k_pad), -2, r_pad))
        b_bank.append(pad_dim(pad_last(B, r_pad), -2, n_pad))
    return torch.stack(a_bank).contiguous(), torch.stack(b_bank).contiguous()


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(
            f"{what}: stageml_b200 runs on CUDA tensors (sm_100a) and has no CPU fallback; got {t.device}")


def require_16bit(t: torch.Tensor, what: str) -> None:
    if t.dtype not in (torch.bfloat16, torch.float16):
        raise RuntimeError(f"{what}: the sm_100a tensor-core path computes in bf16 or fp16; got {t.dtype}")
