"""Expert parallelism on 2 GPUs over NCCL (skipped with fewer GPUs).

Each rank runs its own tokens through EPMoELayer (experts sharded across the
two GPUs, all-to-all dispatch and return) and through the single-GPU layer
with all experts; without shared experts the two are bit-identical because
every routed row is computed independently and combined in the same slot
order.
"""

import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime

        import torch.distributed as dist

        import stageml_b200.ops as ops
        from stageml_b200.expert_parallel import EPMoELayer
        from stageml_b200.workloads import MoEConfig, _Gen, make_moe_workload, sample_tenants

        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        results = []
        for ns in (0, 1):
            cfg = MoEConfig("ep", T=300, H=256, I=384, E=4, k=2, n_shared=ns, n_tenants=5, rank=16,
                            tenant_dist="uniform")
            w = make_moe_workload(cfg, device=dev, gen_device="cpu", seed=0)
            g = _Gen(50 + rank, "cpu", dev)
            x = g.normal((cfg.T, cfg.H), 1.0, torch.bfloat16)
            ten = torch.tensor(sample_tenants(cfg.T, cfg.n_tenants, "uniform", seed=50 + rank), dtype=torch.int32,
                               device=dev)
            layer = EPMoELayer.from_full_weights(cfg, w, rank=rank, world=world)
            y_ep = layer(x, ten)
            y_1 = ops.moe_forward(x, w["gate_up"], w["down"], router_w=w["router_w"], k=cfg.k, n_shared=ns,
                                  tenant_ids=ten, n_tenants=cfg.n_tenants, rank=cfg.bank_rank, lora_a13=w["lora_a13"],
                                  lora_b13=w["lora_b13"], lora_a2=w["lora_a2"], lora_b2=w["lora_b2"],
                                  lora_scale=w["lora_scale"])
            torch.cuda.synchronize()
            rel = ((y_ep.float() - y_1.float()).norm() / y_1.float().norm()).item()
            results.append((ns, bool(torch.equal(y_ep, y_1)), rel))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", results))
    except Exception as exc:
        q.put((rank, "error", f"{exc}\n{traceback.format_exc()[-1500:]}"))


def test_ep_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, status, info = q.get(timeout=300)
            res[rank] = (status, info)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (status, info) in res.items():
        assert status == "ok", info
        for ns, equal, rel in info:
            if ns == 0:
                assert equal, f"rank {rank}: EP differs from single GPU (rel {rel})"
            assert rel < 1e-2, f"rank {rank} n_shared={ns}: rel {rel}"
