"""One-expert top-1 MoE-LoRA layer (a dense SwiGLU MLP with per-row tenants) in token order.

With one expert and top-1 every token is one row of its only expert, so the layer
skips the permutation, the gather and the combine: the shrinks read x and h in
place, the GEMMs take the rows as one group and the down projection writes the
output rows with the routing weight. STAGEML_DIRECT_ROWS=0 keeps the permuted path.
Both run in child processes; both must match the oracle, and every case gives the
same bits either way (each GEMM row and S row is computed on its own).
"""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL16 = 1e-2
HERE = Path(__file__).resolve().parent
MODES = {"direct": {}, "permuted": {"STAGEML_DIRECT_ROWS": "0"}}


def _run(env_extra: dict, out: Path) -> dict:
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, str(HERE / "shrink_modes_child.py"), str(out)], env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def results(tmp_path_factory):
    d = tmp_path_factory.mktemp("direct_rows")
    res = {}
    for m, env in MODES.items():
        res[m] = _run(env, d / f"{m}.pt")
        res[m]["_y"] = torch.load(d / f"{m}.pt")
    return res


@pytest.mark.parametrize("mode", list(MODES))
def test_layer_matches_oracle(results, mode):
    res = results[mode]
    assert res["status"] == 0
    for name, v in res.items():
        if name not in ("status", "_y"):
            assert v["rel_l2"] < TOL16, (mode, name, v)


def test_direct_rows_same_bits_as_permuted(results):
    for name, y in results["permuted"]["_y"].items():
        assert torch.equal(results["direct"]["_y"][name], y), name


def test_direct_rows_drop_bad_ids_and_tenants():
    """A token whose expert id is not 0 or whose tenant is out of range gives a zero
    row and status 110, as the permuted path drops its pair; the other rows are the
    same bits as a call with valid ids."""
    import stageml_b200.ops as ops

    dev = "cuda:0"
    g = torch.Generator(device="cpu").manual_seed(5)
    T, H, I, nT, r = 300, 256, 384, 4, 16
    rnd = lambda *shape, s=1.0: (torch.randn(*shape, generator=g) * s).to(device=dev, dtype=torch.bfloat16)
    x, gu, dn = rnd(T, H), rnd(1, 2 * I, H, s=H ** -0.5), rnd(1, H, I, s=I ** -0.5)
    kw = dict(n_tenants=nT, rank=r, lora_a13=rnd(nT, 1, 2 * r, H, s=H ** -0.5), lora_b13=rnd(nT, 1, 2 * I, r, s=0.25),
              lora_a2=rnd(nT, 1, r, I, s=I ** -0.5), lora_b2=rnd(nT, 1, H, r, s=0.25),
              lora_scale=torch.full((nT,), 2.0, device=dev))
    ten = (torch.arange(T, device=dev, dtype=torch.int32) % (nT + 1)) - 1
    w = torch.rand(T, 1, generator=g).to(dev) + 0.5
    ids = torch.zeros(T, 1, dtype=torch.int64, device=dev)
    ops.take_status(torch.empty(1, device=dev))
    y_ok = ops.moe_forward(x, gu, dn, topk_ids=ids, topk_weights=w, tenant_ids=ten, **kw)
    assert ops.take_status(torch.empty(1, device=dev)) == 0
    bad_ids, bad_ten = ids.clone(), ten.clone()
    bad_ids[5, 0] = 1
    bad_ids[77, 0] = -3
    bad_ten[9] = nT + 7
    y = ops.moe_forward(x, gu, dn, topk_ids=bad_ids, topk_weights=w, tenant_ids=bad_ten, **kw)
    assert ops.take_status(torch.empty(1, device=dev)) == 110
    dropped = torch.zeros(T, dtype=torch.bool, device=dev)
    dropped[[5, 77, 9]] = True
    assert torch.count_nonzero(y[dropped]) == 0
    assert torch.equal(y[~dropped], y_ok[~dropped])
