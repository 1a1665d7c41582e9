"""Test configuration: the `gpu` marker and helpers shared by the test files."""

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a); run with -m gpu")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture
def golden():
    return load_golden


def oracle_moe_tokens(sel, ids, wts, tenant_ids, x, expert_weights, lora_slices=None, lora_scale=None, *,
                      n_routed: int, n_shared: int = 0):
    """The oracle MoE-LoRA layer output of the tokens `sel` only, one expert at a time.

    A token's output is the sum over its experts (routed slots, then always-on shared
    experts with weight 1) of the oracle's single-expert layer, so the full-size
    layers are checked without holding every expert's weights on the host at once.
    expert_weights(e) -> (gate_up [2I, H], down [H, I]); lora_slices(e) -> the four
    bank slices [nT, 1, ...] of expert e, or None without LoRA. ids / wts [T, k].
    """
    from oracle import moe as omoe

    sel = np.asarray(sel)
    ids_s = np.asarray(ids)[sel]
    wts_s = np.asarray(wts, dtype=np.float64)[sel]
    ten_s = np.asarray(tenant_ids)[sel]
    xs = np.asarray(x, dtype=np.float64)
    out = np.zeros((sel.size, xs.shape[1]))
    experts = sorted(set(int(e) for e in np.unique(ids_s))) + list(range(n_routed, n_routed + n_shared))
    for e in experts:
        if e < n_routed:
            rows, slots = np.nonzero(ids_s == e)
            weight = wts_s[rows, slots]
        else:
            rows, weight = np.arange(sel.size), np.ones(sel.size)
        gu, dn = expert_weights(e)
        lo = {} if lora_slices is None else dict(zip(("lora_a13", "lora_b13", "lora_a2", "lora_b2"), lora_slices(e)))
        y = omoe.moe_forward(xs[rows], gu[None], dn[None], np.zeros((rows.size, 1), np.int64), weight[:, None],
                             tenant_ids=ten_s[rows], lora_scale=lora_scale, **lo)
        np.add.at(out, rows, y)
    return out
