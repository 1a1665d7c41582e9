"""Benchmark of the StageML MoE-LoRA residual path on B200.

  python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference] [--workload NAME]

One step = one MoE-LoRA FFN layer call (router -> permutation -> SwiGLU experts
with per-token-tenant LoRA on w1/w3/w2 -> combine) over one batch of tokens
already resident in HBM. Metric: layer tokens/s (whole job, all ranks).

N = 1: the Mixtral-shape layer (T=2048, H=4096, I=14336, E=8, top-2, rank-16
LoRA for 32 tenants, bf16). N > 1 (torchrun, one process per GPU, NCCL):
expert parallel -- each rank routes its own 2048 tokens, experts are sharded
E/N per rank with their adapter-bank slices, and routed rows go to their
experts' ranks and back through peer memory over NVLink (this library's
exchange kernels; no NCCL on the data path) (weak scaling: per-GPU work fixed).

--impl reference: the reference's CPU path restated with its own torch operations
(RequestExecutor.dynamic_one, float32; oracle/torch_executor.py, pinned to the
reference's outputs) timed on the host cores on a token sample of the same
workload; under torchrun only rank 0 runs it.

Prints ONE JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}
L2_BYTES = 126 * 1024 * 1024


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            d["source"] = "measured"
            return d
        except Exception:
            pass
    return dict(FALLBACK_PEAKS)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU every ~20 ms (NVML, or nvidia-smi)."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
        0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, int, int]] = []
        self._stop = threading.Event()
        self._t = None
        self.max_mhz = None
        self._nvml = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _poll(self):
        while not self._stop.is_set():
            try:
                if self._nvml:
                    sm = self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM)
                    rs = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                else:
                    out = subprocess.run(["nvidia-smi", "-i", str(self.index), "--query-gpu=clocks.sm,clocks.max.sm",
                                          "--format=csv,noheader,nounits"], capture_output=True, text=True).stdout
                    a, b = out.strip().split(",")[:2]
                    sm, rs = int(a), 0
                    self.max_mhz = int(b)
                self.samples.append((time.time(), int(sm), int(rs)))
            except Exception:
                pass
            self._stop.wait(0.02)

    def start(self):
        self._t = threading.Thread(target=self._poll, daemon=True)
        self._t.start()

    def stop(self) -> dict:
        self._stop.set()
        if self._t:
            self._t.join(timeout=2)
        sms = [s[1] for s in self.samples]
        reasons = set()
        for _, _, rs in self.samples:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        reasons.discard("gpu_idle")
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sms)}


# ------------------------------------------------------------------ helpers
def capi():
    from stageml_b200._native import load_capi

    return load_capi()


def stage_times(lib) -> dict:
    import ctypes

    from stageml_b200.capi import STAGE_NAMES

    n = len(STAGE_NAMES)
    ms = (ctypes.c_float * n)()
    cnt = (ctypes.c_int32 * n)()
    lib.stageml_stage_timer_read(ms, cnt, n)
    return {STAGE_NAMES[i]: {"ms": float(ms[i]), "launches": int(cnt[i])} for i in range(n) if cnt[i] > 0}


def cpu_threads() -> int:
    n = os.cpu_count() or 1
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:
        pass
    return min(n, 64)  # numpy's OpenBLAS build caps at 64 threads


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


# ------------------------------------------------------------------ CPU arm
CPU_PATHS = {
    "torch": "torch restatement of the reference's RequestExecutor.dynamic_one (per (slot, expert): nonzero, "
             "index_select, F.linear on w1/w3/w2 with each tenant's LoRA, index_add_), float32, incl. router",
    "numpy": "numpy/OpenBLAS float32 grouped executor of the oracle, incl. router",
}


def run_cpu_sample(cfg, w, sample_tokens: int, repeats: int, warmup: int, budget_s: float | None = None,
                   impl: str = "torch"):
    """Time a CPU restatement of the reference's executor on `sample_tokens` tokens of the workload;
    returns (tokens_per_s, times). impl "torch": the reference's own torch operations
    (oracle/torch_executor.py, pinned to the reference's outputs); "numpy": the oracle's executor."""
    import numpy as np

    from oracle.moe import MoEExecutorF32
    from oracle.route import route_topk
    from oracle.torch_executor import dynamic_executor

    t0 = time.time()
    f32 = lambda t: None if t is None else t.float().cpu().numpy()

    def weights(name):  # e4m3 weights are dequantised with their per-row scales (q * scale[:, None])
        s = w.get(name + "_scale")
        return f32(w[name]) if s is None else f32(w[name]) * f32(s)[..., None]

    x = f32(w["x"][:sample_tokens])
    gw = f32(w["router_w"])
    ten = w["tenant_ids"][:sample_tokens].cpu().numpy()
    if impl == "torch":
        torch.set_num_threads(cpu_threads())
        tt = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a))
        banks = {n: tt(f32(w[n])) for n in ("lora_a13", "lora_b13", "lora_a2", "lora_b2", "lora_scale")}
        gu, dn, xt, tent = tt(weights("gate_up")), tt(weights("down")), tt(x), tt(ten)
        gwt = tt(gw)

        def step():
            probs = torch.softmax(xt @ gwt.t(), -1)  # make_routing: fp32 logits, softmax, top-k, renormalise
            wts, ids = torch.topk(probs, cfg.k, -1)
            wts = wts / wts.sum(-1, keepdim=True)
            return dynamic_executor(xt, gu, dn, ids, wts, tent, n_shared=cfg.n_shared, **banks)
    else:
        ex = MoEExecutorF32(weights("gate_up"), weights("down"), n_shared=cfg.n_shared, lora_a13=f32(w["lora_a13"]),
                            lora_b13=f32(w["lora_b13"]), lora_a2=f32(w["lora_a2"]), lora_b2=f32(w["lora_b2"]),
                            lora_scale=f32(w["lora_scale"]))

        def step():
            ids, wts, _ = route_topk(x, gw, cfg.k, True)
            return ex(x, ids, wts, ten)
    log(f"cpu arm ({impl}): weights on host in {time.time() - t0:.1f}s; {cpu_threads()} threads, {cpu_model()}")

    for _ in range(warmup):
        step()
    times = []
    for i in range(repeats):
        t = time.perf_counter()
        step()
        times.append(time.perf_counter() - t)
        if budget_s is not None and sum(times) > budget_s and i >= 0:
            break
    return sample_tokens / statistics.median(times), times


def reference_arm(args, cfg, rank: int):
    if rank != 0:
        return
    import numpy as np  # noqa: F401

    from stageml_b200.workloads import make_moe_workload

    torch.cuda.set_device(0)
    w = make_moe_workload(cfg, device="cuda", seed=0)
    sample = args.cpu_sample_tokens
    tps, times = run_cpu_sample(cfg, w, sample, repeats=args.steps, warmup=args.warmup, impl="torch")
    cores = cpu_threads()
    line = {
        "metric": "MoE-LoRA layer tokens/s", "value": round(tps, 3), "unit": "tokens/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup,
        "ms_per_step": round(1000 * statistics.mean(times), 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; shapes of the Mixtral layer)",
        "config": {"workload": cfg.name, "tokens_per_step": sample, "hidden": cfg.H, "intermediate": cfg.I,
                   "experts": cfg.E, "top_k": cfg.k, "lora_rank": cfg.rank, "tenants": cfg.n_tenants},
        "cpu_baseline": {"value": round(tps, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                         "path": CPU_PATHS["torch"],
                         "sample": f"{sample} of {cfg.T} tokens per step (all experts and tenants touched), "
                                   f"{cpu_model()}"},
        "e2e": {"value": round(tps, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def layer_call(ops, cfg, w, x, tenant_ids):
    return ops.moe_forward(x, w["gate_up"], w["down"], router_w=w["router_w"], k=cfg.k, n_shared=cfg.n_shared,
                           renormalize=True, tenant_ids=tenant_ids, n_tenants=cfg.n_tenants, rank=cfg.bank_rank,
                           lora_a13=w["lora_a13"], lora_b13=w["lora_b13"], lora_a2=w["lora_a2"],
                           lora_b2=w["lora_b2"], lora_scale=w["lora_scale"], gate_up_scale=w["gate_up_scale"],
                           down_scale=w["down_scale"])


def ours_arm(args, cfg, rank: int, world: int, local_rank: int):
    import stageml_b200.ops as ops
    from stageml_b200.workloads import make_moe_workload, moe_bytes

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = capi()
    peaks = load_peaks()
    T = args.tokens or cfg.T
    t_gen = time.time()
    layer = None
    if world > 1:
        from stageml_b200.expert_parallel import EPMoELayer

        w = make_moe_workload(cfg, device=dev, seed=0, T=T)  # identical weights on every rank (seed 0)
        x_local = make_moe_workload_tokens(cfg, dev, seed=1000 + rank, T=T)
        w["x"], w["tenant_ids"] = x_local
        layer = EPMoELayer.from_full_weights(cfg, w, rank=rank, world=world)
        call = lambda x, ten: layer(x, ten)
    else:
        w = make_moe_workload(cfg, device=dev, seed=0, T=T)
        call = lambda x, ten: layer_call(ops, cfg, w, x, ten)
    torch.cuda.synchronize()
    log(f"rank {rank}: workload {cfg.name} T={T} ready in {time.time() - t_gen:.1f}s")

    x, ten = w["x"], w["tenant_ids"]
    for _ in range(args.warmup):
        call(x, ten)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()

    # ---- batch-1 latency (p50 over 200 calls, CUDA events), N=1 only; measured before
    # the throughput run, on its own warm-up, like a separate latency benchmark
    batch1 = None
    if world == 1 and not args.skip_batch1:
        xb, tb = x[:1].contiguous(), ten[:1].contiguous()
        for _ in range(10):
            call(xb, tb)
        lat = []
        for _ in range(200):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            call(xb, tb)
            b.record()
            b.synchronize()
            lat.append(a.elapsed_time(b) * 1000.0)
        lat.sort()
        # HBM roofline of the call: the touched experts' weights (distinct top-k ids of
        # the token, plus shared experts), their adapter slices and the row in / out
        ids_b = ops.route_topk(xb, w["router_w"], cfg.k, True)[0]
        n_exp = len(set(ids_b.flatten().tolist())) + cfg.n_shared
        esz = 1 if cfg.weight_dtype == "e4m3" else 2
        b1_bytes = n_exp * 3 * cfg.H * cfg.I * esz + (cfg.k + cfg.n_shared) * moe_bytes(cfg, w, 1)["adapter_per_pair"] + 2 * cfg.H * 2
        t_b1 = b1_bytes / (float(peaks.get("hbm_gbs", 6650.0)) * 1e9) * 1e6
        p50 = lat[len(lat) // 2]
        batch1 = {"p50_us": round(p50, 2), "p95_us": round(lat[int(len(lat) * 0.95)], 2), "samples": len(lat),
                  "roofline": {"bound": "hbm", "bytes": b1_bytes, "experts_touched": n_exp,
                               "t_roof_us": round(t_b1, 2), "frac": round(t_b1 / p50, 4)}}

    # ---- timed region: device-resident inputs. CUDA events around the gate/up GEMM
    # stage only (one event pair per step, on the layer's stream) give the dominant
    # kernel's time from these same steps.
    STAGE_GATE_UP = 3
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.05)
    n0 = lib.stageml_launch_count()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    lib.stageml_stage_timer_read(None, None, 0)  # forget earlier records
    lib.stageml_stage_timer_select(1 << STAGE_GATE_UP)
    lib.stageml_stage_timer_enable(1)
    t_wall = time.perf_counter()
    e0.record()
    for _ in range(args.steps):
        call(x, ten)
    e1.record()
    torch.cuda.synchronize()
    region_s = time.perf_counter() - t_wall
    lib.stageml_stage_timer_enable(0)
    lib.stageml_stage_timer_select(0xFFFFFFFF)
    n1 = lib.stageml_launch_count()
    ms_total = e0.elapsed_time(e1)
    timed_stages = stage_times(lib)
    clocks = sampler.stop()
    # the cost of the two events: short loops with and without them, alternated so that
    # both see the same power state (the GPU leaves its burst clocks within ~0.1 s)
    ms_with = ms_without = 0.0
    lib.stageml_stage_timer_select(1 << STAGE_GATE_UP)
    for rep in range(6):
        on = rep % 2 == 0
        lib.stageml_stage_timer_enable(1 if on else 0)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(5):
            call(x, ten)
        e1.record()
        torch.cuda.synchronize()
        if on:
            ms_with += e0.elapsed_time(e1)
        else:
            ms_without += e0.elapsed_time(e1)
    lib.stageml_stage_timer_enable(0)
    lib.stageml_stage_timer_select(0xFFFFFFFF)
    lib.stageml_stage_timer_read(None, None, 0)
    # stage breakdown from a separate pass (every stage's events stay out of the timed steps)
    stage_steps = min(args.steps, 10)
    lib.stageml_stage_timer_enable(1)
    for _ in range(stage_steps):
        call(x, ten)
    torch.cuda.synchronize()
    lib.stageml_stage_timer_enable(0)
    stages = stage_times(lib)
    if world > 1:
        t = torch.tensor([ms_total, ms_with, ms_without], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_total, ms_with, ms_without = (float(v) for v in t.tolist())
    ms_step = ms_total / args.steps
    value = world * T / (ms_step / 1000.0)

    # ---- end to end: pinned host input -> device -> layer -> host output, every step.
    # As in a serving loop the copies overlap the neighbouring steps' layer calls:
    # step i+1's input is copied in (copy stream) while step i computes, and step
    # i's output is copied out while step i+1 computes (double-buffered).
    x_host = x.cpu().pin_memory()
    ten_host = ten.cpu().pin_memory()
    out_host = [torch.empty((T, cfg.H), dtype=x.dtype).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x) for _ in range(2)]
    ten_dev = [torch.empty_like(ten) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    loaded = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    # as many steps as the timed device-resident region, so that both see the same power state
    e2e_steps = max(3, args.steps)

    def e2e_run(n):
        cur = torch.cuda.current_stream()
        s_in.wait_stream(cur)
        s_out.wait_stream(cur)

        def copy_in(i):
            b = i % 2
            if i >= 2:
                s_in.wait_event(freed[b])  # step i-2 no longer reads this buffer
            with torch.cuda.stream(s_in):
                x_dev[b].copy_(x_host, non_blocking=True)
                ten_dev[b].copy_(ten_host, non_blocking=True)
            loaded[b].record(s_in)

        copy_in(0)
        for i in range(n):
            if i + 1 < n:
                copy_in(i + 1)
            b = i % 2
            cur.wait_event(loaded[b])
            y = call(x_dev[b], ten_dev[b])
            freed[b].record(cur)
            s_out.wait_stream(cur)
            with torch.cuda.stream(s_out):
                out_host[b].copy_(y, non_blocking=True)
            y.record_stream(s_out)
        cur.wait_stream(s_out)
        cur.wait_stream(s_in)

    e2e_run(3)
    torch.cuda.synchronize()
    # The device-resident steps, the event-overhead loops and the stage pass have just
    # held the GPU at its power cap; the end-to-end steps start, like the timed steps
    # did, from an idle GPU (at N = 2, layer-only steps measured right after 20 end-to-end
    # steps take 1.79 ms against 1.51 ms from idle), so the two numbers compare the copies
    # and not the power state.
    time.sleep(0.5)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0.record()
    t_host = time.perf_counter()
    e2e_run(e2e_steps)
    host_submit_ms = (time.perf_counter() - t_host) * 1000.0 / e2e_steps  # host time to issue one step
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = e0.elapsed_time(e1)
    host_io = host_copy_rates(x_host, out_host[0], x_dev[0], x, world, dev) if world > 1 else None
    if host_io is not None:
        host_io["host_submit_ms_per_step"] = round(host_submit_ms, 4)
    if world > 1:
        t = torch.tensor([ms_e2e], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms_e2e = float(t.item())
    e2e_value = world * T / (ms_e2e / e2e_steps / 1000.0)
    h2d = x_host.numel() * x_host.element_size() + ten_host.numel() * ten_host.element_size()
    d2h = out_host[0].numel() * out_host[0].element_size()

    ep_status = ep_parity = None
    if layer is not None:  # collective: every rank releases the exchange buffers
        ep_parity = expert_parallel_parity(ops, cfg, w, layer, x, ten, dev)
        ep_status = layer.take_status()
        layer.close()
    if rank != 0:
        return
    fl = cfg.flops(T)
    dom = "gemm_gate_up"
    dom_ms = timed_stages[dom]["ms"] / max(timed_stages[dom]["launches"], 1) if dom in timed_stages else None
    dom_flops = fl["gate_up"] + 2.0 * T * (cfg.k + cfg.n_shared) * 2 * cfg.I * cfg.rank
    peak = choose_peak(peaks, clocks, region_s)
    achieved = dom_flops / (dom_ms / 1000.0) / 1e12 if dom_ms else None
    by = moe_bytes(cfg, w, T)
    layer_bytes = by["weights"] + by["activations"]
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    t_roof = {kind: max(fl["total"] / (tf * 1e12), layer_bytes / (hbm * 1e9))
              for kind, tf in (("burst", peak["burst"]), ("sustained", peak["sustained"]))}
    # DRAM traffic of one gate/up GEMM launch from a committed ncu capture, or None
    cap = GATE_UP_DRAM_CAPTURE.get(cfg.name) if T == cfg.T and world == 1 else None
    cpu = None
    if world == 1 and not args.skip_cpu:
        try:
            tps, times = run_cpu_sample(cfg, w, args.cpu_sample_tokens, repeats=5, warmup=1, budget_s=15.0,
                                        impl="torch")
            tps_np, times_np = run_cpu_sample(cfg, w, args.cpu_sample_tokens, repeats=3, warmup=1, budget_s=8.0,
                                              impl="numpy")
            cpu = {"value": round(tps, 3), "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
                   "path": CPU_PATHS["torch"],
                   "sample": f"{args.cpu_sample_tokens} of {T} tokens, median of {len(times)} timed calls after 1 "
                             f"warm-up; {cpu_model()}",
                   "numpy_port": {"value": round(tps_np, 3), "unit": "tokens/s", "path": CPU_PATHS["numpy"],
                                  "timed_calls": len(times_np)}}
        except Exception as exc:  # pragma: no cover
            cpu = {"value": None, "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
                   "sample": f"failed: {exc}"}
    line = {
        "metric": "MoE-LoRA layer tokens/s",
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1/fan_in) weights, N(0,1) tokens; no checkpoints available)",
        "config": {"workload": cfg.name, "tokens_per_gpu": T, "global_batch": T * world, "hidden": cfg.H,
                   "intermediate": cfg.I, "experts": cfg.E, "top_k": cfg.k, "lora_rank": cfg.rank,
                   "tenants": cfg.n_tenants, "lora_on": "w1,w3,w2", "router": "in-layer (fp32 logits, softmax, top-2)",
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "ep_transport": layer.transport if layer is not None else None,
                   "l2": f"inputs larger than L2 ({by['weights'] / 1e9:.2f} GB expert weights per step)"},
        "roofline": {"bound": "tensor", "kernel": "grouped gate/up GEMM (tcgen05) + LoRA expand + SwiGLU",
                     "achieved": None if achieved is None else round(achieved, 1), "peak": peak["value"],
                     "unit": "TFLOP/s", "frac": None if achieved is None else round(achieved / peak["value"], 4),
                     "peak_kind": peak["kind"],
                     "frac_burst": None if achieved is None else round(achieved / peak["burst"], 4),
                     "frac_sustained": None if achieved is None else round(achieved / peak["sustained"], 4),
                     "traffic": None if cap is None else cap["bytes"],
                     "traffic_source": None if cap is None else cap["source"],
                     "launch_ms": None if dom_ms is None else round(dom_ms, 4),
                     "launch_ms_source": f"CUDA events around the gate/up stage inside the {args.steps} timed steps",
                     "flops_per_launch": dom_flops,
                     "peak_source": f"{peaks.get('source')} {peak['why']}"},
        "layer_roofline": {"flops": fl["total"], "bytes": layer_bytes, "peak_kind": peak["kind"],
                           "t_roof_ms": round(t_roof[peak["kind"]] * 1000, 4),
                           "frac": round(t_roof[peak["kind"]] * 1000 / ms_step, 4),
                           "frac_burst": round(t_roof["burst"] * 1000 / ms_step, 4),
                           "frac_sustained": round(t_roof["sustained"] * 1000 / ms_step, 4)},
        "timed_region_s": round(region_s, 4),
        "event_overhead": {"frac": round(ms_with / ms_without - 1.0, 5) if ms_without > 0 else None,
                           "how": "3 loops of 5 steps with the gate/up events alternated with 3 without"},
        "stages_ms_per_step": {k: round(v["ms"] / stage_steps, 4) for k, v in stages.items()},
        "stages_source": f"separate pass of {stage_steps} calls with every stage's events",
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps,
                "api": ("torch.ops.stageml.moe_forward" if layer is None else
                        "stageml_b200.expert_parallel.EPMoELayer.__call__ (expert parallel over peer memory)") +
                       " (pinned host in/out, every step's copies timed; they overlap the neighbouring steps' layer "
                       "calls on copy streams, double-buffered)"},
        "gpu_launches": int(n1 - n0),
        "clocks": clocks,
        "batch1_latency": batch1,
        "cpu_baseline": cpu,
    }
    if layer is not None:
        line["ep_status"] = ep_status
        line["ep_parity"] = ep_parity
        line["host_io"] = host_io
    if world == 1 and cfg.name == "mixtral_moe_lora" and not args.skip_configs:
        line["other_configs"] = other_configs(args)
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of one full-size gate/up GEMM launch, from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum of every kernel of the launch), with
# the build it was captured on. It is stale once the GEMM changes after that build.
GATE_UP_DRAM_CAPTURE: dict = {
    "mixtral_moe_lora": {
        "bytes": 2.376832e9 + 0.132748e9,
        "source": "ncu capture of commit 24e4d5a: pair kernel with the odd tiles as half units, 2.510 GB "
                  "(profiles/grouped_gemm_pair_mixtral.md)",
    },
}


def gpu_numa_node(dev) -> int | None:
    try:
        bus = torch.cuda.get_device_properties(dev).pci_bus_id if hasattr(
            torch.cuda.get_device_properties(dev), "pci_bus_id") else None
        if bus is None:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(dev.index if hasattr(dev, "index") else int(dev))
            bus = pynvml.nvmlDeviceGetPciInfo(h).busId
            bus = bus.decode() if isinstance(bus, bytes) else bus
        bus = bus.lower()
        if bus.count(":") == 2 and len(bus.split(":")[0]) == 8:
            bus = bus[4:]
        return int(open(f"/sys/bus/pci/devices/{bus}/numa_node").read().strip())
    except Exception:
        return None


def host_copy_rates(x_host, out_host, x_dev, y_dev, world: int, dev) -> dict:
    """Per-rank host<->device copy rates of one step's input and output, every rank copying at
    the same time (as in the end-to-end loop); collective. Also where the rank's pinned memory
    and GPU sit (NUMA nodes) and which CPUs the process may run on."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    rates = []
    for src, dst in ((x_host, x_dev), (y_dev, out_host)):
        for _ in range(2):
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        e0.record()
        for _ in range(5):
            dst.copy_(src, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        rates.append(5 * src.numel() * src.element_size() / (e0.elapsed_time(e1) / 1e3) / 1e9)
    t = torch.tensor(rates, device=dev)
    lo, hi = t.clone(), t.clone()
    torch.distributed.all_reduce(lo, op=torch.distributed.ReduceOp.MIN)
    torch.distributed.all_reduce(hi, op=torch.distributed.ReduceOp.MAX)
    try:
        cpus = sorted(os.sched_getaffinity(0))
        cpu_span = f"{len(cpus)} cpus {cpus[0]}-{cpus[-1]}"
    except Exception:
        cpu_span = None
    return {"h2d_gbs_min": round(float(lo[0]), 2), "h2d_gbs_max": round(float(hi[0]), 2),
            "d2h_gbs_min": round(float(lo[1]), 2), "d2h_gbs_max": round(float(hi[1]), 2),
            "all_ranks_copying": True, "rank0_gpu_numa": gpu_numa_node(dev), "rank0_cpus": cpu_span}


def choose_peak(peaks: dict, clocks: dict, region_s: float) -> dict:
    """The bf16 peak a kernel timed in this run is held to: the burst figure while the
    SM clock stayed at its maximum over a short timed region, the sustained
    (power-capped, seconds-long) figure otherwise."""
    burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    sustained = float(peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"]))
    sm, mx = clocks.get("sm_mhz"), clocks.get("sm_max_mhz")
    at_max = bool(sm and mx and sm >= 0.97 * float(mx))
    if at_max and region_s < 1.0:
        return {"kind": "burst", "value": burst, "burst": burst, "sustained": sustained,
                "why": f"bf16_tflops (burst): median SM clock {sm} of max {mx} MHz over a {region_s:.3f} s region"}
    return {"kind": "sustained", "value": sustained, "burst": burst, "sustained": sustained,
            "why": f"bf16_tflops_sustained: median SM clock {sm} of max {mx} MHz over a {region_s:.3f} s region"}


def expert_parallel_parity(ops, cfg, w, layer, x, ten, dev, sample: int = 64) -> dict:
    """Each rank checks its first `sample` tokens of one expert-parallel call against the
    single-GPU layer holding every expert (same weights on every rank). Collective:
    every rank takes part. Returns the max rel-L2 over ranks and how many sampled
    rows came out bit-identical."""
    y_ep = layer(x, ten)
    n = min(sample, x.shape[0])
    y_one = layer_call(ops, cfg, w, x[:n].contiguous(), ten[:n].contiguous())
    a, b = y_ep[:n].float(), y_one.float()
    rel = (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b).clamp_min(1e-30)).reshape(1)
    same = (y_ep[:n] == y_one).all(dim=1).sum().to(torch.float32).reshape(1)
    rel_max, same_sum = rel.clone(), same.clone()
    torch.distributed.all_reduce(rel_max, op=torch.distributed.ReduceOp.MAX)
    torch.distributed.all_reduce(same_sum, op=torch.distributed.ReduceOp.SUM)
    world = torch.distributed.get_world_size()
    return {"max_rel_l2": float(rel_max.item()), "rows_checked": n * world, "rows_bit_identical": int(same_sum.item()),
            "against": "ops.moe_forward on one GPU with all experts, first tokens of every rank", "tolerance": 1e-2}


# ------------------------------------------------------------------ other configurations
def _timed(fn, steps: int, warmup: int, lib=None):
    """Device time of `steps` calls after `warmup` calls; returns (ms per call, stage times, launches)."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    if lib is not None:
        n0 = lib.stageml_launch_count()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    stages, launches = {}, None
    if lib is not None:
        launches = int(lib.stageml_launch_count() - n0)
        # per-stage breakdown (ms per call) from a separate pass, outside the timed calls
        n_st = min(steps, 10)
        lib.stageml_stage_timer_enable(1)
        for i in range(n_st):
            fn(i)
        torch.cuda.synchronize()
        lib.stageml_stage_timer_enable(0)
        stages = {k: {"ms": v["ms"] / n_st, "launches": 1} for k, v in stage_times(lib).items()}
    return e0.elapsed_time(e1) / steps, stages, launches


def _graph_timed(fn, reps: int, replays: int = 5):
    """Device time per call of `reps` calls captured in one CUDA graph (host submission
    overhead excluded), replayed `replays` times after one warm-up replay; ms per call."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                fn(i)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(replays):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / (replays * reps)


_COLLECT: list | None = None  # when a list, result lines of dense_arm are appended to it instead of printed


def _line(metric, value, unit, steps, warmup, ms, hib, dtype, config, **extra):
    d = {"metric": metric, "value": value, "unit": unit, "n_gpus": 1, "steps": steps, "warmup": warmup,
         "ms_per_step": round(ms, 5), "higher_is_better": hib, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
         "data": "synthetic (seeded; shapes of the configuration)", "config": config}
    d.update(extra)
    if _COLLECT is not None:
        _COLLECT.append(d)
    else:
        print(json.dumps(d), flush=True)


# The other configurations, measured after the headline layer in a default 1-GPU run and
# summarised in its line (each with its own clock record).
OTHER_CONFIGS = ("single_lora", "adapter_bank", "llama_block", "fine_grained_fp8_moe_lora")


def other_configs(args) -> dict:
    global _COLLECT
    out = {}
    for name in OTHER_CONFIGS:
        sub = argparse.Namespace(**vars(args))
        sub.workload, sub.steps, sub.warmup = name, min(args.steps, 20), 3
        _COLLECT = []
        t0 = time.time()
        try:
            dense_arm(sub)
            d = _COLLECT[-1]
            keep = ("metric", "value", "unit", "ms_per_step", "steps", "roofline", "layer_roofline", "fold",
                    "folded_latency_us", "folded_roofline", "stages_ms_per_step", "clocks", "config", "value_source",
                    "api_call_ms")
            out[name] = {k: d[k] for k in keep if k in d}
        except Exception as exc:  # one configuration failing must not lose the headline line
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        finally:
            _COLLECT = None
            torch.cuda.empty_cache()
        out[name]["wall_s"] = round(time.time() - t0, 1)
    return out


def dense_arm(args):
    """Configurations 1-3 and the fine-grained MoE layer with bf16 weights, one JSON line each.

    These are the parity configurations beside the headline MoE-LoRA layer; the driver's
    headline line is the default workload.
    """
    import numpy as np

    import stageml_b200.ops as ops
    from stageml_b200 import workloads as wl

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = capi()
    peaks = load_peaks()
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    name = args.workload
    sampler = ClockSampler(0)
    sampler.start()
    if name == "single_lora":
        # x[1,4096] fp32, W[4096,4096] ([in,out]), rank 16, scale 2; 4 rotating weight sets (268 MB > L2)
        sets = [wl.make_single_lora(seed=s, device=dev) for s in range(4)]
        folded = [ops.lora_fold(s["W"], s["A"], s["B"], s["scale"], 1) for s in sets]
        ms_dyn, st_dyn, n_dyn = _timed(lambda i: ops.lora_gemv_f32(sets[i % 4]["x"], sets[i % 4]["W"], sets[i % 4]["A"],
                                                                    sets[i % 4]["B"], sets[i % 4]["scale"]),
                                       args.steps, args.warmup, lib)
        ms_fold, _, _ = _timed(lambda i: ops.lora_gemv_f32(sets[i % 4]["x"], folded[i % 4]), args.steps, args.warmup)
        # the stage-0 fold W' = W + s A B itself: reads W, writes W' (4 B per element each)
        sc1 = torch.full((1,), float(sets[0]["scale"]), dtype=torch.float32, device=dev)
        sc4 = [torch.full((1,), float(st["scale"]), dtype=torch.float32, device=dev) for st in sets]
        # device time per call with the host out of the loop (calls captured in a CUDA graph)
        g_dyn = _graph_timed(lambda i: ops.lora_gemv_f32(sets[i % 4]["x"], sets[i % 4]["W"], sets[i % 4]["A"],
                                                         sets[i % 4]["B"], sets[i % 4]["scale"]), 40)
        g_fold = _graph_timed(lambda i: ops.lora_gemv_f32(sets[i % 4]["x"], folded[i % 4]), 40)
        g_f = _graph_timed(lambda i: ops.lora_fold(sets[i % 4]["W"], sets[i % 4]["A"], sets[i % 4]["B"], sc4[i % 4],
                                                   1), 20)
        ms_f, _, n_f = _timed(lambda i: ops.lora_fold(sets[i % 4]["W"], sets[i % 4]["A"], sets[i % 4]["B"], sc1, 1),
                              args.steps, args.warmup, lib)
        fold_bytes = 2 * 4 * 4096 * 4096 + 2 * 4 * 4096 * 16
        byt = 4 * 4096 * 4096 + 2 * 4 * 4096 * 16 + 8 * 4096
        ms_k = st_dyn.get("gemv", {}).get("ms", 0) / max(st_dyn.get("gemv", {}).get("launches", 1), 1)
        s0 = sets[0]
        f = lambda t: t.cpu().numpy()
        from oracle.lora import single_lora

        t0 = time.perf_counter()
        reps = 0
        while time.perf_counter() - t0 < 2.0:
            single_lora(f(s0["x"]), f(s0["W"]), f(s0["A"]), f(s0["B"]), s0["scale"], dtype=np.float32)
            reps += 1
        cpu_us = (time.perf_counter() - t0) / reps * 1e6
        _line("single LoRA linear latency (dynamic x W + s (x A) B)", round(g_dyn * 1000, 3), "us", args.steps,
              args.warmup, g_dyn, False, "f32",
              {"workload": "single_lora", "x": [1, 4096], "W": [4096, 4096], "rank": 16, "scale": 2.0,
               "l2": "4 rotating weight sets, 268 MB > L2"},
              value_source="device time per call: 40 calls (4 rotating weight sets) in one CUDA graph",
              eager_latency_us=round(ms_dyn * 1000, 3), folded_latency_us=round(g_fold * 1000, 3),
              eager_folded_latency_us=round(ms_fold * 1000, 3),
              folded_roofline={"bytes": 4 * 4096 * 4096 + 8 * 4096,
                               "achieved_gbs": round((4 * 4096 * 4096 + 8 * 4096) / (g_fold / 1e3) / 1e9, 1),
                               "frac": round((4 * 4096 * 4096 + 8 * 4096) / (g_fold / 1e3) / 1e9 / hbm, 4)},
              gpu_launches=n_dyn, clocks=sampler.stop(),
              fold={"kernel": "fold_f32_vec_kernel (fp32, [in,out] layout)", "us": round(g_f * 1000, 3),
                    "bytes": fold_bytes, "achieved_gbs": round(fold_bytes / (g_f / 1e3) / 1e9, 1),
                    "frac": round(fold_bytes / (g_f / 1e3) / 1e9 / hbm, 4), "eager_us": round(ms_f * 1000, 3),
                    "launches": n_f, "timing": "CUDA graph of 20 folds, 4 rotating weight sets"},
              roofline={"bound": "hbm", "kernel": "gemv_partial_kernel + reduce (dynamic form)",
                        "achieved": round(byt / (g_dyn / 1e3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(byt / (g_dyn / 1e3) / 1e9 / hbm, 4), "traffic": None,
                        "stage_timer_ms": round(ms_k, 5)},
              cpu_baseline={"value": round(cpu_us, 2), "unit": "us", "cores": cpu_threads(), "kind": "port",
                            "sample": "the same call, numpy float32"})
    elif name == "adapter_bank":
        from stageml_b200.adapter_bank import AdapterSpec
        from stageml_b200.adapter_cache import StageMLCostBasedAdapterCache

        w = wl.make_adapter_bank(seed=0, device=dev)
        ads = [AdapterSpec(f"adapter_{i}", w["A"][i], w["B"][i], w["scale"]) for i in range(w["A"].shape[0])]
        names = [f"adapter_{i}" for i in w["adapter_ids"]]
        cached = [f"adapter_{i}" for i in w["folded"]]
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        layers = []
        e0.record()
        layers.append(StageMLCostBasedAdapterCache(w["W"], ads, cached_adapter_names=cached))
        e1.record()
        torch.cuda.synchronize()
        fold_ms = e0.elapsed_time(e1)
        layers += [StageMLCostBasedAdapterCache(w["W"] * (1 + 1e-3 * j), ads, cached_adapter_names=cached)
                   for j in range(1, 3)]  # 3 layers x 302 MB of weights rotate past L2
        # the stage-0 fold alone: the 8 cached adapters folded into W (bf16) in one batched launch,
        # W read once and 8 W' written; 3 rotating base weights
        idx = torch.tensor([int(c.split("_")[1]) for c in cached], device=dev)
        A8, B8 = w["A"][idx].contiguous(), w["B"][idx].contiguous()
        sc8 = torch.full((len(cached),), float(w["scale"]), dtype=torch.float32, device=dev)
        Ws = [w["W"], layers[1].weight, layers[2].weight]
        ms_f, _, n_f = _timed(lambda i: ops.lora_fold(Ws[i % 3], A8, B8, sc8, 0), args.steps, args.warmup, lib)
        g_f = _graph_timed(lambda i: ops.lora_fold(Ws[i % 3], A8, B8, sc8, 0), 12)
        fold_bytes = 4096 * 4096 * 2 * (1 + len(cached)) + (A8.numel() + B8.numel()) * 2
        # the layer's op with its row groups / tenants resident on the device (what the class passes
        # to it each call), and the class call itself (adapter names -> index tensors on the host)
        lay0 = layers[0]
        grp_t = torch.tensor([lay0.cached_name_to_index[nm] + 1 if nm in lay0.cached_name_to_index else 0
                              for nm in names], dtype=torch.int32, device=dev)
        ten_t = torch.tensor([-1 if nm in lay0.cached_name_to_index else lay0.adapter_index[nm] for nm in names],
                             dtype=torch.int32, device=dev)

        def op_call(i):
            lay = layers[i % 3]
            return ops.lora_linear(w["x"], lay.weight_bank, bias=lay.bias, row_group=grp_t, row_tenant=ten_t,
                                   n_tenants=len(lay.adapter_order), rank=lay.rank_pad, lora_a=lay.lora_a,
                                   lora_b=lay.lora_b, lora_scale=lay.lora_scale)

        ref_y = layers[0](w["x"], names)
        assert torch.equal(op_call(0), ref_y), "op call differs from the class call"
        ms, st, n = _timed(op_call, args.steps, args.warmup, lib)
        ms_api, _, _ = _timed(lambda i: layers[i % 3](w["x"], names), args.steps, args.warmup)
        byt = 4096 * 4096 * 2 * (1 + len(cached)) + 2 * 256 * 4096 * 2
        _line("multi-tenant LoRA bank tokens/s (64 adapters, top-8 folded)", round(256 / (ms / 1e3), 1), "tokens/s",
              args.steps, args.warmup, ms, True, "bf16",
              {"workload": "adapter_bank", "tokens": 256, "dim": 4096, "adapters": 64, "rank": 16,
               "folded": len(cached), "l2": "3 rotating layers"},
              stages_ms_per_step={k: round(v["ms"] / max(v["launches"], 1), 4) for k, v in st.items()},
              api_call_ms=round(ms_api, 5),
              value_source="ops.lora_linear with the row groups / tenants resident; api_call_ms: "
                           "StageMLCostBasedAdapterCache.forward from adapter-name lists",
              stage0_fold_ms=round(fold_ms, 4), gpu_launches=n, clocks=sampler.stop(),
              fold={"kernel": "fold_mma_kernel (bf16, 8 adapters batched, W broadcast)", "us": round(g_f * 1000, 3),
                    "bytes": fold_bytes, "achieved_gbs": round(fold_bytes / (g_f / 1e3) / 1e9, 1),
                    "frac": round(fold_bytes / (g_f / 1e3) / 1e9 / hbm, 4), "eager_us": round(ms_f * 1000, 3),
                    "launches": n_f, "timing": "CUDA graph of 12 folds, 3 rotating base weights"},
              roofline={"bound": "hbm", "kernel": "grouped GEMM over [W, W'_1..8] + tensor-core LoRA expand",
                        "achieved": round(byt / (ms / 1e3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(byt / (ms / 1e3) / 1e9 / hbm, 4), "traffic": None})
    elif name == "llama_block":
        blk = wl.make_llama_block(seed=0, device=dev)
        P = blk["proj"]
        r, nT = 16, 16
        ten = blk["row_tenant"]
        sc = torch.full((nT,), blk["scale"], dtype=torch.float32, device=dev)
        # MLP = one-expert SwiGLU MoE layer: gate_up = [W_gate; W_up], LoRA A13 = [A_gate; A_up], B13 = [B_gate; B_up]
        gu = torch.cat([P["gate"]["W"], P["up"]["W"]], 0)[None].contiguous()
        dn = P["down"]["W"][None].contiguous()
        a13 = torch.cat([P["gate"]["A"], P["up"]["A"]], 1)[:, None].contiguous()
        b13 = torch.cat([P["gate"]["B"], P["up"]["B"]], 1)[:, None].contiguous()
        a2 = P["down"]["A"][:, None].contiguous()
        b2 = P["down"]["B"][:, None].contiguous()
        M = blk["x"].shape[0]
        ids = torch.zeros(M, 1, dtype=torch.int32, device=dev)
        ones = torch.ones(M, 1, dtype=torch.float32, device=dev)

        def step(i):
            outs = [ops.lora_linear(blk["x"] if p != "o" else blk["x_o"], P[p]["W"][None], row_tenant=ten, n_tenants=nT,
                                    rank=r, lora_a=P[p]["A"], lora_b=P[p]["B"], lora_scale=sc) for p in "qkvo"]
            outs.append(ops.moe_forward(blk["x"], gu, dn, topk_ids=ids, topk_weights=ones, tenant_ids=ten,
                                        n_tenants=nT, rank=r, lora_a13=a13, lora_b13=b13, lora_a2=a2, lora_b2=b2,
                                        lora_scale=sc))
            return outs

        ms, st, n = _timed(step, args.steps, args.warmup, lib)
        clocks = sampler.stop()
        pk = choose_peak(peaks, clocks, ms * args.steps / 1e3)
        fl = 2.0 * M * (4 * 4096 * 4096 + 3 * 4096 * 11008) + 2.0 * M * r * (4 * 2 * 4096 + 3 * (4096 + 11008))
        _line("LLaMA-7B block projections with LoRA tokens/s", round(M / (ms / 1e3), 1), "tokens/s", args.steps,
              args.warmup, ms, True, "fp16",
              {"workload": "llama_block", "tokens": M, "projections": "q,k,v,o,gate,up,down", "rank": r,
               "tenants": nT, "attention": "excluded"},
              stages_ms_per_step={k: round(v["ms"] / max(v["launches"], 1), 4) for k, v in st.items()},
              gpu_launches=n, clocks=clocks,
              roofline={"bound": "tensor", "kernel": "all grouped GEMMs of the block", "flops": fl,
                        "achieved": round(fl / (ms / 1e3) / 1e12, 1), "peak": pk["value"], "unit": "TFLOP/s",
                        "frac": round(fl / (ms / 1e3) / 1e12 / pk["value"], 4), "peak_kind": pk["kind"],
                        "frac_burst": round(fl / (ms / 1e3) / 1e12 / pk["burst"], 4),
                        "frac_sustained": round(fl / (ms / 1e3) / 1e12 / pk["sustained"], 4), "traffic": None,
                        "peak_source": pk["why"]})
    elif name in ("fine_grained_moe_lora_bf16", "fine_grained_fp8_moe_lora"):
        cfg = wl.MoEConfig(name, T=8192, H=2048, I=1408, E=64, k=6, n_shared=2, n_tenants=128, rank=8,
                           tenant_dist="zipf", weight_dtype="e4m3" if "fp8" in name else "bf16")
        w = wl.make_moe_workload(cfg, device=dev, seed=0)
        ms, st, n = _timed(lambda i: layer_call(ops, cfg, w, w["x"], w["tenant_ids"]), args.steps, args.warmup, lib)
        clocks = sampler.stop()
        pk = choose_peak(peaks, clocks, ms * args.steps / 1e3)
        fl = cfg.flops()
        _line(f"fine-grained MoE-LoRA layer tokens/s ({cfg.weight_dtype} weights)", round(cfg.T / (ms / 1e3), 1),
              "tokens/s", args.steps, args.warmup, ms, True, "bf16",
              {"workload": cfg.name, "tokens": cfg.T, "hidden": 2048, "intermediate": 1408, "experts": 64, "top_k": 6,
               "shared_experts": 2, "tenants": 128, "lora_rank": 8,
               "weights": cfg.weight_dtype},
              stages_ms_per_step={k: round(v["ms"] / max(v["launches"], 1), 4) for k, v in st.items()},
              gpu_launches=n, clocks=clocks,
              layer_roofline={"flops": fl["total"], "peak_kind": pk["kind"],
                              "t_roof_ms": round(fl["total"] / (pk["value"] * 1e12) * 1e3, 4),
                              "frac": round(fl["total"] / (pk["value"] * 1e12) * 1e3 / ms, 4),
                              "frac_burst": round(fl["total"] / (pk["burst"] * 1e12) * 1e3 / ms, 4),
                              "frac_sustained": round(fl["total"] / (pk["sustained"] * 1e12) * 1e3 / ms, 4),
                              "peak_source": pk["why"]})
    elif name == "request_stream":
        # the reference system benchmark's request stream (128 requests x 16 tokens over 512
        # token rows, 16 Zipf(1.2) tenants in bursts of 8 on 8 rank-16 w1 adapters, memory-budget
        # materialization) on Mixtral-shape experts: the whole stream as one layer call
        from stageml_b200.executor import RequestExecutor, make_workload_plan, run_sequence
        from stageml_b200.moe_lora_layers import MoEAdapterSpec

        H, I, E, k, nA, r, Tav = 4096, 14336, 8, 2, 8, 16, 512
        g = wl._Gen(0, "cuda", dev)
        hidden = g.normal((Tav, H), 1.0, torch.bfloat16)
        gate_up = g.normal_stacked(E, (2 * I, H), H ** -0.5, torch.bfloat16)
        down = g.normal_stacked(E, (H, I), I ** -0.5, torch.bfloat16)
        router_w = g.normal((E, H), H ** -0.5, torch.float32)
        ids, wts, _ = ops.route_topk(hidden, router_w, k, True)
        ads = [MoEAdapterSpec(f"adapter_{i}", g.normal_stacked(E, (r, H), H ** -0.5, torch.bfloat16),
                              g.normal_stacked(E, (I, r), r ** -0.5, torch.bfloat16), 2.0) for i in range(nA)]
        folded_bytes = E * I * H * 2
        plan = make_workload_plan(num_requests=128, num_tenants=16, num_adapters=nA, tokens_available=Tav,
                                  tokens_per_request=16, distribution="zipf", zipf_alpha=1.2, burst_size=8,
                                  materialization_policy="memory_budget", materialize_top_k=4,
                                  materialize_min_requests=2, memory_budget_mb=2048.0,
                                  memory_per_adapter_bytes=folded_bytes, seed=17)
        ex = RequestExecutor(gate_up, down, ads, plan.materialized_adapter_ids)
        toks = sum(q.end - q.start for q in plan.requests)
        ms, st, n = _timed(lambda i: run_sequence(ex, plan, hidden, ids, wts, "batched"), args.steps, args.warmup,
                           lib)
        per = {}
        for mode in ("dynamic", "bta"):
            ms_m, _, n_m = _timed(lambda i: run_sequence(ex, plan, hidden, ids, wts, mode), max(3, args.steps // 10),
                                  2, lib)
            per[mode] = {"ms_per_stream": round(ms_m, 4), "tokens_per_s": round(toks / (ms_m / 1e3), 1),
                         "gpu_launches": n_m}
        _line("request stream tokens/s (128 requests x 16 tokens, Mixtral experts, w1 adapters)",
              round(toks / (ms / 1e3), 1), "tokens/s", args.steps, args.warmup, ms, True, "bf16",
              {"workload": "request_stream", "requests": len(plan.requests), "tokens_per_request": 16,
               "tokens": toks, "token_rows": Tav, "hidden": H, "intermediate": I, "experts": E, "top_k": k,
               "tenants": 16, "adapters": nA, "rank": r, "materialized": sorted(plan.materialized_adapter_ids),
               "mode": "batched: the whole stream as one layer call"},
              per_request_modes=per, stage0_fold_ms=round(ex.compile_time_ms, 3), gpu_launches=n,
              clocks=sampler.stop())
    else:
        raise SystemExit(f"unknown workload {name}")


DENSE_WORKLOADS = ("single_lora", "adapter_bank", "llama_block", "fine_grained_moe_lora_bf16", "request_stream")


def make_moe_workload_tokens(cfg, dev, seed: int, T: int):
    from stageml_b200.workloads import _Gen, sample_tenants

    g = _Gen(seed, "cuda", dev)
    x = g.normal((T, cfg.H), 1.0, torch.bfloat16)
    ten = torch.tensor(sample_tenants(T, cfg.n_tenants, cfg.tenant_dist, cfg.alpha, seed=seed), dtype=torch.int32,
                       device=dev)
    return x, ten


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="mixtral_moe_lora")
    ap.add_argument("--tokens", type=int, default=0, help="tokens per GPU per step (default: the workload's)")
    ap.add_argument("--cpu-sample-tokens", type=int, default=256)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-batch1", action="store_true")
    ap.add_argument("--skip-configs", action="store_true",
                    help="do not measure the other configurations after the headline layer")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        log("note: warm-up raised to the minimum of 3 steps")
        args.warmup = 3

    sys.path.insert(0, str(ROOT))
    from stageml_b200.workloads import MOE_CONFIGS

    if args.workload in DENSE_WORKLOADS:
        dense_arm(args)
        return
    cfg = MOE_CONFIGS[args.workload]
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, cfg, rank)
        return
    if world > 1:
        import datetime

        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local_rank))
    try:
        ours_arm(args, cfg, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
