"""Parity through the C ABI itself (ctypes, no torch dispatcher): the calls a
non-torch host would make, with torch used only to own device memory."""

import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_l2
from oracle import moe as omoe
from oracle import permute as operm
from stageml_b200 import capi

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def lib():
    from stageml_b200._native import load_capi

    torch.cuda.init()
    return load_capi()


def p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def f64(t):
    return t.detach().float().cpu().numpy().astype(np.float64)


def test_moe_forward_through_c_abi(lib):
    g = torch.Generator().manual_seed(0)
    T, H, I, E, k, nT, r = 300, 256, 384, 4, 2, 3, 16
    bf = torch.bfloat16
    x = torch.randn(T, H, generator=g).to(DEV, bf)
    gu = (torch.randn(E, 2 * I, H, generator=g) / 16).to(DEV, bf)
    dn = (torch.randn(E, H, I, generator=g) / 20).to(DEV, bf)
    gw = (torch.randn(E, H, generator=g) / 16).to(DEV)
    a13 = (torch.randn(nT, E, 2 * r, H, generator=g) / 16).to(DEV, bf)
    b13 = (torch.randn(nT, E, 2 * I, r, generator=g) / 4).to(DEV, bf)
    a2 = (torch.randn(nT, E, r, I, generator=g) / 20).to(DEV, bf)
    b2 = (torch.randn(nT, E, H, r, generator=g) / 4).to(DEV, bf)
    sc = torch.tensor([0.5, 1.0, 2.0], device=DEV)
    ten = torch.randint(-1, nT, (T,), generator=g, dtype=torch.int32).to(DEV)
    out = torch.empty(T, H, device=DEV, dtype=bf)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    # keep the permutation in caller memory to check it too
    P = T * k
    cap = lib.stageml_plan_rows_cap(P, E)
    bufs = {n: torch.empty(cap, dtype=torch.int32, device=DEV) for n in ("row_token", "row_tenant", "row_pair")}
    bufs["row_weight"] = torch.empty(cap, dtype=torch.float32, device=DEV)
    bufs["pair_row"] = torch.empty(P, dtype=torch.int32, device=DEV)
    bufs["tile_group"] = torch.empty(cap // 128, dtype=torch.int32, device=DEV)
    bufs["group_offsets"] = torch.empty(E + 1, dtype=torch.int32, device=DEV)
    bufs["group_counts"] = torch.empty(E, dtype=torch.int32, device=DEV)
    bufs["num_tiles"] = torch.empty(1, dtype=torch.int32, device=DEV)
    plan = capi.MoePlan(**{n: t.data_ptr() for n, t in bufs.items()}, rows_cap=cap)
    a = capi.MoeArgs(T=T, H=H, I=I, E=E, k=k, n_shared=0, act_dtype=capi.BF16, weight_dtype=capi.BF16,
                     x=x.data_ptr(), router_w=gw.data_ptr(), renormalize=1, tenant_ids=ten.data_ptr(), n_tenants=nT,
                     rank=r, gate_up=gu.data_ptr(), down=dn.data_ptr(), lora_a13=a13.data_ptr(),
                     lora_b13=b13.data_ptr(), lora_a2=a2.data_ptr(), lora_b2=b2.data_ptr(), lora_scale=sc.data_ptr(),
                     out=out.data_ptr(), status=status.data_ptr(), plan_out=ctypes.addressof(plan))
    need = lib.stageml_moe_workspace_bytes(ctypes.byref(a))
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    rc = lib.stageml_moe_forward(ctypes.byref(a), p(ws), need, stream())
    capi.check(lib, rc, "stageml_moe_forward")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # routing with the same C ABI
    ids = torch.empty(T, k, dtype=torch.int32, device=DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=DEV)
    logits = torch.empty(T, E, dtype=torch.float32, device=DEV)
    capi.check(lib, lib.stageml_route_topk(p(x), capi.BF16, p(gw), T, H, E, k, 1, p(logits), p(ids), p(w), stream()),
               "route")
    torch.cuda.synchronize()
    ref = omoe.moe_forward(f64(x), f64(gu), f64(dn), ids.cpu().numpy(), w.cpu().numpy(), tenant_ids=ten.cpu().numpy(),
                           lora_a13=f64(a13), lora_b13=f64(b13), lora_a2=f64(a2), lora_b2=f64(b2),
                           lora_scale=sc.cpu().numpy())
    assert rel_l2(f64(out), ref) < 1e-2
    pref = operm.permute(ids.cpu().numpy(), w.cpu().numpy(), ten.cpu().numpy(), E, 0, nT)
    nt = int(bufs["num_tiles"].item())
    assert nt == pref["num_tiles"]
    np.testing.assert_array_equal(bufs["row_pair"][: nt * 128].cpu().numpy(), pref["row_pair"])
    np.testing.assert_array_equal(bufs["pair_row"].cpu().numpy(), pref["pair_row"])
    # the torch op gives the identical bits
    import stageml_b200.ops as ops

    y2 = ops.moe_forward(x, gu, dn, router_w=gw, k=k, tenant_ids=ten, n_tenants=nT, rank=r, lora_a13=a13,
                         lora_b13=b13, lora_a2=a2, lora_b2=b2, lora_scale=sc)
    assert torch.equal(y2, out)


def test_residual_moe_through_c_abi(lib):
    g = torch.Generator().manual_seed(1)
    T, H, I, E, k = 129, 128, 256, 5, 2
    x = torch.randn(T, H, generator=g).to(DEV, torch.float16)
    gu = (torch.randn(E, 2 * I, H, generator=g) / 11).to(DEV, torch.float16)
    dn = (torch.randn(E, H, I, generator=g) / 16).to(DEV, torch.float16)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(DEV)
    w = torch.rand(T, k, generator=g).to(DEV)
    out = torch.empty(T, H, device=DEV, dtype=torch.float16)
    need = lib.stageml_residual_moe_workspace_bytes(T, H, I, E, k)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    rc = lib.stageml_residual_moe(p(x), p(gu), p(dn), p(w), capi.F32, p(ids), capi.I64, T, H, I, E, k, capi.F16,
                                  p(out), None, p(ws), need, stream())
    capi.check(lib, rc, "stageml_residual_moe")
    torch.cuda.synchronize()
    ref = omoe.fallback_moe(f64(x), f64(gu), f64(dn), w.cpu().numpy(), ids.cpu().numpy())
    assert rel_l2(f64(out), ref) < 1e-2


def test_fold_and_gemv_through_c_abi(lib):
    g = torch.Generator().manual_seed(2)
    din, dout, r = 512, 384, 16
    x = torch.randn(2, din, generator=g).to(DEV)
    W = (torch.randn(din, dout, generator=g) / 20).to(DEV)
    A = (torch.randn(din, r, generator=g) / 20).to(DEV)
    B = (torch.randn(r, dout, generator=g) / 4).to(DEV)
    sc = torch.tensor([2.0], device=DEV)
    Wf = torch.empty_like(W)
    capi.check(lib, lib.stageml_lora_fold(p(W), p(A), p(B), p(sc), 1, din, dout, r, 1, 0, 0, 0, capi.F32, p(Wf),
                                          stream()), "fold")
    y = torch.empty(2, dout, device=DEV)
    need = lib.stageml_lora_gemv_f32_workspace_bytes(2, din, dout, r)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    capi.check(lib, lib.stageml_lora_gemv_f32(p(x), p(W), p(A), p(B), 2.0, 2, din, dout, r, p(y), p(ws), need,
                                              stream()), "gemv")
    yf = torch.empty(2, dout, device=DEV)
    capi.check(lib, lib.stageml_lora_gemv_f32(p(x), p(Wf), None, None, 0.0, 2, din, dout, 0, p(yf), p(ws), need,
                                              stream()), "gemv folded")
    torch.cuda.synchronize()
    ref = f64(x) @ f64(W) + 2.0 * (f64(x) @ f64(A)) @ f64(B)
    assert rel_l2(f64(y), ref) < 1e-5
    assert rel_l2(f64(yf), ref) < 1e-5


def test_stage_timer_and_launch_counter(lib):
    import stageml_b200.ops as ops

    x = torch.randn(64, 64, device=DEV, dtype=torch.bfloat16)
    W = torch.randn(1, 64, 64, device=DEV, dtype=torch.bfloat16)
    n0 = lib.stageml_launch_count()
    lib.stageml_stage_timer_enable(1)
    ops.lora_linear(x, W)
    lib.stageml_stage_timer_enable(0)
    ms = (ctypes.c_float * 10)()
    cnt = (ctypes.c_int32 * 10)()
    assert lib.stageml_stage_timer_read(ms, cnt, 10) == 0
    assert cnt[7] == 1 and ms[7] > 0.0  # the GEMM stage
    assert lib.stageml_launch_count() - n0 == 1
