"""Expert-parallel host logic on CPU with gloo, world size 2.

The dispatch / exchange / combine of stageml_b200.expert_parallel.EPMoELayer is
run with the oracle's router and expert MLP injected in place of the CUDA
kernels; every rank's output must equal the single-process oracle layer for
its own tokens. A rank that fails before the exchange must make the other rank
fail with an error within the process-group timeout, not hang.
"""

import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(E, ns, H, I, nT, r, seed=0):
    rng = np.random.default_rng(seed)
    Et = E + ns
    return dict(gate_up=rng.standard_normal((Et, 2 * I, H)) / H ** 0.5, down=rng.standard_normal((Et, H, I)) / I ** 0.5,
                router=rng.standard_normal((E, H)) / H ** 0.5,
                a13=rng.standard_normal((nT, Et, 2 * r, H)) / H ** 0.5, b13=rng.standard_normal((nT, Et, 2 * I, r)),
                a2=rng.standard_normal((nT, Et, r, I)) / I ** 0.5, b2=rng.standard_normal((nT, Et, H, r)),
                scale=rng.uniform(0.5, 2, nT))


def _worker(rank, world, port, cfg, q):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime

        import torch
        import torch.distributed as dist

        from oracle import moe as omoe
        from oracle import route as oroute
        from stageml_b200.expert_parallel import EPMoELayer

        torch.set_num_threads(1)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        E, ns, H, I, k, nT, r, T = (cfg[n] for n in ("E", "ns", "H", "I", "k", "nT", "r", "T"))
        W = _weights(E, ns, H, I, nT, r)
        rng = np.random.default_rng(100 + rank)
        x = rng.standard_normal((T, H))
        if cfg.get("skew"):
            x = x + 5 * W["router"][0]  # pull every token towards expert 0 (owned by rank 0)
        ten = rng.integers(-1, nT, T)
        E_loc = E // world
        own = list(range(rank * E_loc, (rank + 1) * E_loc)) + list(range(E, E + ns))

        def route_fn(xt):
            ids, w, _ = oroute.route_topk(xt.numpy(), W["router"], k, True)
            return torch.from_numpy(ids), torch.from_numpy(w)

        lw = {n: W[n][own] for n in ("gate_up", "down")}
        ll = {n: W[n][:, own] for n in ("a13", "b13", "a2", "b2")}

        def local_fn(xr, expert, tenant, weight):
            y = omoe.moe_forward(xr.numpy(), lw["gate_up"], lw["down"], expert.numpy()[:, None],
                                 weight.numpy()[:, None], tenant_ids=tenant.numpy(), lora_a13=ll["a13"],
                                 lora_b13=ll["b13"], lora_a2=ll["a2"], lora_b2=ll["b2"], lora_scale=W["scale"])
            return torch.from_numpy(y)

        def shared_fn(xt, tenant):
            ids0 = np.zeros((xt.shape[0], 0), dtype=np.int64)
            y = omoe.moe_forward(xt.numpy(), lw["gate_up"], lw["down"], ids0, None, tenant_ids=tenant.numpy(),
                                 n_shared=ns, lora_a13=ll["a13"], lora_b13=ll["b13"], lora_a2=ll["a2"],
                                 lora_b2=ll["b2"], lora_scale=W["scale"])
            return torch.from_numpy(y)

        def combine_fn(y_back, pair_row, T_, k_):
            return y_back[pair_row.long()].view(T_, k_, -1).sum(1)

        if cfg.get("fail_rank") == rank:
            raise RuntimeError("injected failure before the exchange")
        layer = EPMoELayer(E=E, k=k, n_shared=ns, H=H, I=I, rank=rank, world=world, gate_up_local=None,
                           down_local=None, router_w=None, route_fn=route_fn, local_fn=local_fn, shared_fn=shared_fn,
                           combine_fn=combine_fn)
        y = layer(torch.from_numpy(x), torch.from_numpy(ten))
        ids, w, _ = oroute.route_topk(x, W["router"], k, True)
        ref = omoe.moe_forward(x, W["gate_up"], W["down"], ids, w, tenant_ids=ten, n_shared=ns, lora_a13=W["a13"],
                               lora_b13=W["b13"], lora_a2=W["a2"], lora_b2=W["b2"], lora_scale=W["scale"])
        err = float(np.abs(y.numpy() - ref).max() / np.abs(ref).max())
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", err))
    except Exception as exc:  # report to the parent instead of hanging
        q.put((rank, "error", f"{type(exc).__name__}: {exc}\n{traceback.format_exc()[-800:]}"))


def _run(cfg, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, info = q.get(timeout=timeout)
            results[rank] = (status, info)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


BASE = dict(E=4, ns=0, H=16, I=24, k=2, nT=3, r=4, T=37)


@pytest.mark.parametrize("cfg", [BASE, dict(BASE, ns=1, T=20), dict(BASE, skew=True, T=30), dict(BASE, T=1)])
def test_ep_matches_single_process_oracle(cfg):
    res = _run(cfg)
    assert set(res) == {0, 1}
    for rank, (status, info) in res.items():
        assert status == "ok", info
        assert info < 1e-12, f"rank {rank}: max rel err {info}"


def test_ep_peer_failure_is_detected_not_hung():
    res = _run(dict(BASE, fail_rank=1), timeout=90)
    assert res[1][0] == "error" and "injected failure" in res[1][1]
    assert res[0][0] == "error"  # rank 0's exchange fails (peer gone / timeout) instead of blocking forever


def test_ep_op_is_registered_with_a_fake_and_no_cpu_kernel():
    from torch._subclasses.fake_tensor import FakeTensorMode

    import stageml_b200.expert_parallel  # noqa: F401  (defines the op)

    op = torch.ops.stageml.ep_moe_lora_forward
    assert str(op.default._schema) == "stageml::ep_moe_lora_forward(Tensor x, Tensor tenant_ids, int layer) -> Tensor"
    with FakeTensorMode():
        y = op(torch.empty(5, 8, dtype=torch.bfloat16), torch.empty(5, dtype=torch.int32), 1)
        assert y.shape == (5, 8) and y.dtype == torch.bfloat16
    with pytest.raises(NotImplementedError, match="CPU"):  # no CPU path
        op(torch.zeros(2, 8), torch.zeros(2, dtype=torch.int32), 1)
