"""Expert parallelism on 2 GPUs (skipped with fewer GPUs).

Each rank runs its own tokens through EPMoELayer (experts sharded across the
two GPUs) and through the single-GPU layer with all experts. Both transports
are checked: "peer" (rows stored into the other GPU's memory through CUDA IPC,
epoch flags, no host-side split sizes) and "collective" (NCCL all-to-all).
Without shared experts the peer-transport result is bit-identical to the
single-GPU layer whenever both run the tensor-memory GEMM (more than 16 routed
rows): every routed row is computed by the same kernels and combined in the
same slot order. Everything else -- shared experts (different sum order), tiny
batches or small receives that take the weight-streaming GEMM, the collective
transport -- is checked at rel-L2 <= 1e-2.
Several calls per layer exercise the reuse of the exchange buffers across
epochs, with a different token count on each rank; one case routes almost every
token to rank 0's experts.
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
        cases = [dict(ns=0, rank=16), dict(ns=1, rank=16), dict(ns=0, rank=0), dict(ns=0, rank=16, skew=True)]
        for case in cases:
            ns = case["ns"]
            cfg = MoEConfig("ep", T=300, H=256, I=384, E=4, k=2, n_shared=ns, n_tenants=5, rank=case["rank"],
                            tenant_dist="uniform")
            w = make_moe_workload(cfg, device=dev, gen_device="cpu", seed=0)
            layers = {t: EPMoELayer.from_full_weights(cfg, w, rank=rank, world=world, transport=t)
                      for t in ("peer", "collective")}
            lora = {}
            if cfg.rank:
                lora = dict(n_tenants=cfg.n_tenants, rank=cfg.rank, lora_a13=w["lora_a13"], lora_b13=w["lora_b13"],
                            lora_a2=w["lora_a2"], lora_b2=w["lora_b2"], lora_scale=w["lora_scale"])
            for call, T in enumerate((300 - 100 * rank, 123 + 50 * rank, 1 + rank)):
                g = _Gen(50 + 7 * call + rank, "cpu", dev)
                x = g.normal((T, cfg.H), 1.0, torch.bfloat16)
                if case.get("skew"):  # every token's top-1 is expert 0 (owned by rank 0)
                    x = x + (5.0 * w["router_w"][0] / w["router_w"][0].norm()).to(x.dtype)
                ten = torch.tensor(sample_tenants(T, cfg.n_tenants, "uniform", seed=50 + call + rank),
                                   dtype=torch.int32, device=dev)
                y_1 = ops.moe_forward(x, w["gate_up"], w["down"], router_w=w["router_w"], k=cfg.k, n_shared=ns,
                                      tenant_ids=ten if cfg.rank else None, **lora)
                outs = {t: layer(x, ten) for t, layer in layers.items()}
                # the same call through the dispatcher
                outs["op"] = torch.ops.stageml.ep_moe_lora_forward(x, ten, layers["peer"].register())
                torch.cuda.synchronize()
                rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()
                exact = ns == 0 and T * cfg.k > 16
                for t, y in outs.items():
                    results.append((str(case), t, call, exact and t in ("peer", "op"), bool(torch.equal(y, y_1)),
                                    rel(y, y_1)))
                results.append((str(case), "peer_vs_collective", call, False, False, rel(outs["peer"], outs["collective"])))
            results.append((str(case), "status", -1, True, layers["peer"].take_status() == 0 and ops.take_status(x) == 0,
                            0.0))
            for layer in layers.values():
                layer.close()
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
            rank, status, info = q.get(timeout=600)
            res[rank] = (status, info)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (status, info) in res.items():
        assert status == "ok", info
        for case, what, call, exact, equal, rel in info:
            if what == "status":
                assert equal, f"rank {rank} {case}: nonzero device status"
            elif exact:
                assert equal, f"rank {rank} {case} {what} call {call}: EP differs from single GPU (rel {rel})"
            else:
                assert rel < 1e-2, f"rank {rank} {case} {what} call {call}: rel {rel}"


def _worker_one(port, q):
    """World size 1: the exchange kernels with this rank as the only peer, through the layer
    and through torch.ops.stageml.ep_moe_lora_forward."""
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        import datetime

        import torch.distributed as dist

        import stageml_b200.ops as ops
        from stageml_b200.expert_parallel import EPMoELayer
        from stageml_b200.workloads import MoEConfig, make_moe_workload

        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60), device_id=dev)
        cfg = MoEConfig("ep1", T=200, H=256, I=256, E=4, k=2, n_shared=0, n_tenants=3, rank=16, tenant_dist="uniform")
        w = make_moe_workload(cfg, device=dev, gen_device="cpu", seed=1)
        lora = dict(n_tenants=cfg.n_tenants, rank=cfg.rank, lora_a13=w["lora_a13"], lora_b13=w["lora_b13"],
                    lora_a2=w["lora_a2"], lora_b2=w["lora_b2"], lora_scale=w["lora_scale"])
        y_1 = ops.moe_forward(w["x"], w["gate_up"], w["down"], router_w=w["router_w"], k=cfg.k,
                              tenant_ids=w["tenant_ids"], **lora)
        results = []
        for t in ("peer", "collective"):
            layer = EPMoELayer.from_full_weights(cfg, w, rank=0, world=1, transport=t)
            for _ in range(2):
                y = torch.ops.stageml.ep_moe_lora_forward(w["x"], w["tenant_ids"], layer.register())
                y_l = layer(w["x"], w["tenant_ids"])
                torch.cuda.synchronize()
                rel = ((y.float() - y_1.float()).norm() / y_1.float().norm()).item()
                results.append((t, bool(torch.equal(y, y_l)), rel, layer.take_status()))
            layer.close()
        dist.destroy_process_group()
        q.put(("ok", results))
    except Exception as exc:
        q.put(("error", f"{exc}\n{traceback.format_exc()[-1500:]}"))


def test_ep_op_on_one_gpu_matches_single_gpu_layer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    proc = ctx.Process(target=_worker_one, args=(_free_port(), q))
    proc.start()
    try:
        status, info = q.get(timeout=600)
    finally:
        proc.join(timeout=60)
        if proc.is_alive():
            proc.kill()
    assert status == "ok", info
    for transport, same_as_layer, rel, dev_status in info:
        assert same_as_layer, transport
        assert rel < 1e-2, (transport, rel)
        assert dev_status == 0, transport
