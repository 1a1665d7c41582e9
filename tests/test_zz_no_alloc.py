"""The allocation-free fp32 single-LoRA GEMV, through the C ABI.

stageml_lora_gemv_f32_noalloc serves callers of this library that cannot
allocate device memory where they run the layer (a plugin with no allocator of
its own, a serving loop that must not call cudaMalloc/cudaFree, a host with a
fixed memory arena): its scratch is a static array inside the library instead
of a caller workspace. This test checks, on two calls in a row, that it gives
the same result as the workspace entry point stageml_lora_gemv_f32 (rel-L2
within the 1e-5 fp32 tolerance of the other tests), and that a shape too large
for the static scratch is refused with an error. The file is named to be
collected last, and it needs no state from other tests.
"""

import ctypes

import numpy as np
import pytest
import torch

from stageml_b200 import capi

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _rel(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_noalloc_gemv_matches_workspace_entry_point():
    from stageml_b200._native import load_capi

    torch.cuda.init()
    lib = load_capi()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = torch.Generator().manual_seed(0)
    M, din, dout, r, s = 1, 4096, 4096, 16, 2.0  # the config-1 single-LoRA shape
    x = torch.randn(M, din, generator=g).to(DEV)
    W = (torch.randn(din, dout, generator=g) / din ** 0.5).to(DEV)
    A = (torch.randn(din, r, generator=g) / din ** 0.5).to(DEV)
    B = (torch.randn(r, dout, generator=g) / r ** 0.5).to(DEV)

    need = lib.stageml_lora_gemv_f32_workspace_bytes(M, din, dout, r)
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    y_ref = torch.empty(M, dout, device=DEV)
    rc = lib.stageml_lora_gemv_f32(_ptr(x), _ptr(W), _ptr(A), _ptr(B), s, M, din, dout, r, _ptr(y_ref), _ptr(ws), need,
                                   stream)
    capi.check(lib, rc, "stageml_lora_gemv_f32")

    for _ in range(2):  # the second call reuses the static scratch left by the first
        y = torch.full((M, dout), float("nan"), device=DEV)
        rc = lib.stageml_lora_gemv_f32_noalloc(_ptr(x), _ptr(W), _ptr(A), _ptr(B), s, M, din, dout, r, _ptr(y), stream)
        capi.check(lib, rc, "stageml_lora_gemv_f32_noalloc")
        torch.cuda.synchronize()
        assert _rel(y, y_ref) <= 1e-5

    # the folded form (A = B = NULL) through the same scratch
    yf = torch.empty(M, dout, device=DEV)
    capi.check(lib, lib.stageml_lora_gemv_f32_noalloc(_ptr(x), _ptr(W), None, None, 0.0, M, din, dout, 0, _ptr(yf),
                                                      stream), "noalloc folded")
    torch.cuda.synchronize()
    assert _rel(yf, x @ W) <= 1e-5

    # a shape whose partial sums do not fit the static scratch (16 rows x 300,000 fp32 output
    # columns need more than 16 MiB) is refused before any launch: nothing is read or written
    wide = 300_000
    assert lib.stageml_lora_gemv_f32_workspace_bytes(16, din, wide, 0) > 16 << 20
    big = torch.empty(16, din, device=DEV)
    out = torch.empty(16, wide, device=DEV)
    rc = lib.stageml_lora_gemv_f32_noalloc(_ptr(big), _ptr(W), None, None, 0.0, 16, din, wide, 0, _ptr(out), stream)
    assert rc == capi.ERR_INVALID_ARG
    assert b"static scratch" in lib.stageml_last_error()
