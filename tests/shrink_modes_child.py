"""Child process of test_gpu_shrink_modes.py, test_gpu_pack_rank8.py and
test_gpu_direct_rows.py: runs LoRA
layers under the kernel choices in its environment (STAGEML_SHRINK, STAGEML_GEMM_PAIRS,
STAGEML_PACK_RANK8, STAGEML_DIRECT_ROWS, each read once per process by the library), prints, per case, the rel-L2 error against the oracle as one JSON line
and saves the outputs to the path given as its argument."""

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


def moe_case(T, H, I, E, k, nT, r, ns=0, dtype=torch.bfloat16, seed=0, zipf=False, caller_weights=False):
    import stageml_b200.ops as ops

    rng = np.random.default_rng(seed)
    Et = E + ns
    x = rand((T, H), 1.0, dtype, seed)
    gu = rand((Et, 2 * I, H), H ** -0.5, dtype, seed + 1)
    dn = rand((Et, H, I), I ** -0.5, dtype, seed + 2)
    rw = rand((E, H), H ** -0.5, torch.float32, seed + 3)
    if zipf:
        p = 1.0 / np.arange(1, nT + 1) ** 1.1
        ten_np = rng.choice(nT, T, p=p / p.sum()).astype(np.int32)
        ten_np[rng.random(T) < 0.05] = -1
    else:
        ten_np = rng.integers(-1, nT, T).astype(np.int32)
    kw = dict(tenant_ids=torch.from_numpy(ten_np).to(DEV), n_tenants=nT, rank=r,
              lora_scale=torch.from_numpy(rng.uniform(0.5, 2.0, nT).astype(np.float32)).to(DEV),
              lora_a13=rand((nT, Et, 2 * r, H), H ** -0.5, dtype, seed + 4),
              lora_b13=rand((nT, Et, 2 * I, r), r ** -0.5, dtype, seed + 5),
              lora_a2=rand((nT, Et, r, I), I ** -0.5, dtype, seed + 6),
              lora_b2=rand((nT, Et, H, r), r ** -0.5, dtype, seed + 7))
    if caller_weights:  # the caller's expert ids and routing weights instead of the router
        ids, _, _ = ops.route_topk(x, rw, k, True)
        w = torch.from_numpy(rng.uniform(0.25, 1.5, (T, k)).astype(np.float32)).to(DEV)
        y = ops.moe_forward(x, gu, dn, topk_ids=ids, topk_weights=w, n_shared=ns, **kw)
    else:
        y = ops.moe_forward(x, gu, dn, router_w=rw, k=k, n_shared=ns, **kw)
        ids, w, _ = ops.route_topk(x, rw, k, True)
    ref = omoe.moe_forward(f64(x), f64(gu), f64(dn), ids.cpu().numpy(), w.cpu().numpy(), tenant_ids=ten_np,
                           n_shared=ns, lora_a13=f64(kw["lora_a13"]), lora_b13=f64(kw["lora_b13"]),
                           lora_a2=f64(kw["lora_a2"]), lora_b2=f64(kw["lora_b2"]), lora_scale=f64(kw["lora_scale"]))
    return y, ref


def linear_case(M, K, N, nT, r, dtype=torch.bfloat16, seed=0):
    """Direct rows (one weight group): the shrink reads the caller's rows in place, in
    their own order, so a 128-row tile holds up to 128 distinct tenants."""
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
    return y, ref


CASES = {
    # 40 tenants: up to 40 per tile, three units of 16 slots in the rank-16 h shrink, two in the x shrink
    "moe_r16_40_tenants": lambda: moe_case(T=600, H=512, I=768, E=4, k=2, nT=40, r=16),
    # rank 8 (R = 8: two tenants per 16 columns), fp16, a shared expert, Zipf tenants
    "moe_r8_f16_shared": lambda: moe_case(T=700, H=384, I=640, E=4, k=2, nT=24, r=8, ns=1, dtype=torch.float16,
                                          seed=3, zipf=True),
    # rank 32 (R = 64 for the packed w1|w3 shrink), K not a multiple of the 512-wide slice
    "moe_r32_ragged_k": lambda: moe_case(T=500, H=320, I=576, E=3, k=2, nT=9, r=32, seed=7),
    # rank 8 with 60 tenants: ~45 runs per tile (past the 32 the GEMMs copy up front), odd and even counts
    "moe_r8_60_tenants": lambda: moe_case(T=900, H=256, I=384, E=4, k=2, nT=60, r=8, seed=17),
    # one expert, top-1 (a dense SwiGLU MLP): rows stay in token order, 650 rows (a partial last tile)
    "moe_e1_router": lambda: moe_case(T=650, H=512, I=704, E=1, k=1, nT=6, r=16, seed=19),
    # one expert with the caller's ids and routing weights, rank 8, fp16
    "moe_e1_caller_weights_r8": lambda: moe_case(T=520, H=384, I=512, E=1, k=1, nT=5, r=8, dtype=torch.float16,
                                                 seed=23, caller_weights=True),
    # direct rows in caller order: 1100 rows (a partial last tile), 150 tenants, rank 8
    "linear_r8_150_tenants": lambda: linear_case(M=1100, K=1024, N=512, nT=150, r=8, seed=11),
    # direct rows, rank 32, K = 1000 (a partial last K block)
    "linear_r32_k1000": lambda: linear_case(M=700, K=1000, N=384, nT=12, r=32, seed=13),
}


def main():
    out, ys = {}, {}
    for name, fn in CASES.items():
        y, ref = fn()
        torch.cuda.synchronize()
        out[name] = {"rel_l2": rel_l2(f64(y), ref)}
        ys[name] = y.float().cpu()
    torch.save(ys, sys.argv[1])
    import stageml_b200.ops as ops

    out["status"] = int(ops.take_status(torch.empty(1, device=DEV)))
    print(json.dumps(out))


if __name__ == "__main__":
    main()
