"""Child process of test_gpu_odd_tiles.py: runs grouped GEMM cases whose groups end in
an odd 128-row tile under the STAGEML_ODD_TILES mode set in its environment (read
once per process by the library) and prints, per case, the rel-L2 error against the
oracle and a digest of the output bits as one JSON line."""

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
sys.path.insert(0, str(Path(__file__).resolve().parent))

from conftest import rel_l2  # noqa: E402
from oracle import moe as omoe  # noqa: E402

DEV = "cuda:0"


def rand(shape, scale, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(device=DEV, dtype=dtype)


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def moe_case(T, H, I, E, k, nT, r, ns=0, dtype=torch.bfloat16, seed=0):
    import stageml_b200.ops as ops

    rng = np.random.default_rng(seed)
    Et = E + ns
    x = rand((T, H), 1.0, dtype, seed)
    gu = rand((Et, 2 * I, H), H ** -0.5, dtype, seed + 1)
    dn = rand((Et, H, I), I ** -0.5, dtype, seed + 2)
    rw = rand((E, H), H ** -0.5, torch.float32, seed + 3)
    kw = {}
    if nT:
        ten = torch.from_numpy(rng.integers(-1, nT, T).astype(np.int32)).to(DEV)
        kw = dict(tenant_ids=ten, n_tenants=nT, rank=r, lora_scale=torch.from_numpy(
            rng.uniform(0.5, 2.0, nT).astype(np.float32)).to(DEV),
                  lora_a13=rand((nT, Et, 2 * r, H), H ** -0.5, dtype, seed + 4),
                  lora_b13=rand((nT, Et, 2 * I, r), r ** -0.5, dtype, seed + 5),
                  lora_a2=rand((nT, Et, r, I), I ** -0.5, dtype, seed + 6),
                  lora_b2=rand((nT, Et, H, r), r ** -0.5, dtype, seed + 7))
    y = ops.moe_forward(x, gu, dn, router_w=rw, k=k, n_shared=ns, **kw)
    ids, w, _ = ops.route_topk(x, rw, k, True)
    g = lambda n: None if kw.get(n) is None else f64(kw[n])
    ref = omoe.moe_forward(f64(x), f64(gu), f64(dn), ids.cpu().numpy(), w.cpu().numpy(),
                           tenant_ids=None if not nT else kw["tenant_ids"].cpu().numpy(), n_shared=ns,
                           lora_a13=g("lora_a13"), lora_b13=g("lora_b13"), lora_a2=g("lora_a2"),
                           lora_b2=g("lora_b2"), lora_scale=g("lora_scale"))
    counts = torch.bincount(ids.flatten().long(), minlength=E).tolist()
    return y, ref, counts


def linear_case(M, K, N, nT, r, dtype=torch.bfloat16, seed=0):
    import stageml_b200.ops as ops

    rng = np.random.default_rng(seed)
    x = rand((M, K), 1.0, dtype, seed + 31)
    W = rand((1, N, K), K ** -0.5, dtype, seed + 32)
    ten = rng.integers(-1, nT, M).astype(np.int32)
    A = rand((nT, r, K), K ** -0.5, dtype, seed + 34)
    B = rand((nT, N, r), r ** -0.5, dtype, seed + 35)
    sc = torch.from_numpy(rng.uniform(0.5, 2, nT).astype(np.float32)).to(DEV)
    y = ops.lora_linear(x, W, row_tenant=torch.from_numpy(ten).to(DEV), n_tenants=nT, rank=r, lora_a=A, lora_b=B,
                        lora_scale=sc)
    ref = f64(x) @ f64(W)[0].T
    m = ten >= 0
    s = np.einsum("mk,mrk->mr", f64(x)[m], f64(A)[ten[m]]) * sc.cpu().numpy()[ten[m]][:, None]
    ref[m] += np.einsum("mr,mnr->mn", s, f64(B)[ten[m]])
    return y, ref, [M]


CASES = {
    # ~350 routed rows per expert: three 128-row tiles, one pair + one odd tile each; LoRA on all projections
    "moe_lora_bf16": lambda: moe_case(T=700, H=512, I=512, E=4, k=2, nT=2, r=16),
    # no LoRA, fp16, a partial last column tile (I = 576) and a shared expert
    "moe_plain_f16": lambda: moe_case(T=700, H=512, I=576, E=4, k=2, nT=0, r=0, ns=1, dtype=torch.float16),
    # rank 8 with a shared expert (routed experts ~600 rows: five tiles each)
    "moe_rank8": lambda: moe_case(T=900, H=512, I=512, E=3, k=2, nT=3, r=8, ns=1, seed=5),
    # direct rows: 384 rows = one tile pair + one odd tile
    "linear_lora": lambda: linear_case(M=384, K=512, N=768, nT=2, r=16),
}


def main():
    out = {}
    for name, fn in CASES.items():
        y, ref, counts = fn()
        torch.cuda.synchronize()
        out[name] = {"rel_l2": rel_l2(f64(y), ref), "sha": hashlib.sha256(y.view(torch.int16).cpu().numpy().tobytes()).hexdigest(),
                     "rows": counts}
    import stageml_b200.ops as ops

    out["status"] = int(ops.take_status(torch.empty(1, device=DEV)))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
