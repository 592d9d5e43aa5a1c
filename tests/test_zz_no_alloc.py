"""The allocation-free RMSNorm + in_proj entry point, called through the C ABI.

nt_rmsnorm_in_proj_noalloc serves callers that cannot allocate device memory
when they run the block (for example serving runtimes that reserve HBM once at
start-up and forbid cudaMalloc afterwards): it keeps its scratch in a device
array owned by the library instead of a caller workspace.  Its results must
match nt_rmsnorm_in_proj, which takes a caller-allocated workspace, call after
call, since every call reuses the same scratch array.  This file is collected
last so that a failing run that stops at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _abi_call_noalloc(L, x, gamma, W, dtype_code):
    M, dm = x.shape
    di = W.shape[0] // 2
    h = torch.empty(M, di, dtype=x.dtype, device=DEV)
    gate = torch.empty_like(h)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.nt_rmsnorm_in_proj_noalloc(dtype_code, M, dm, di, ctypes.c_void_p(x.data_ptr()),
                                      ctypes.c_void_p(gamma.data_ptr()), ctypes.c_void_p(W.data_ptr()),
                                      ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(gate.data_ptr()), stream)
    assert rc == 0, L.nt_last_error()
    return h, gate


def _abi_call_workspace(L, x, gamma, W, dtype_code):
    M, dm = x.shape
    di = W.shape[0] // 2
    h = torch.empty(M, di, dtype=x.dtype, device=DEV)
    gate = torch.empty_like(h)
    nbytes = L.nt_rmsnorm_in_proj_workspace_bytes(dtype_code, M, dm, di)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.nt_rmsnorm_in_proj(dtype_code, M, dm, di, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(gamma.data_ptr()),
                              ctypes.c_void_p(W.data_ptr()), ctypes.c_void_p(h.data_ptr()),
                              ctypes.c_void_p(gate.data_ptr()), ctypes.c_void_p(ws.data_ptr()), nbytes, stream)
    assert rc == 0, L.nt_last_error()
    return h, gate


@pytest.mark.parametrize("dtype,code,tol", [(torch.bfloat16, 1, dict(rtol=1.6e-2, atol=1e-2)),
                                            (torch.float32, 0, dict(rtol=1e-4, atol=1e-5))])
def test_noalloc_matches_workspace_entry_point_twice(dtype, code, tol):
    from neuratensor_b200 import native
    L = native.load()
    g = torch.Generator(device=DEV).manual_seed(123)
    M, dm, di = 4096, 640, 1280
    W = (torch.randn(2 * di, dm, generator=g, device=DEV) / dm ** 0.5).to(dtype)
    gamma = (torch.rand(dm, generator=g, device=DEV) + 0.5).to(dtype)
    for call in range(2):   # the second call reuses the scratch left by the first
        x = (torch.randn(M, dm, generator=g, device=DEV) * (0.5 + call)).to(dtype)
        h0, g0 = _abi_call_workspace(L, x, gamma, W, code)
        h1, g1 = _abi_call_noalloc(L, x, gamma, W, code)
        torch.cuda.synchronize()
        np.testing.assert_allclose(h1.float().cpu().numpy(), h0.float().cpu().numpy(), **tol)
        np.testing.assert_allclose(g1.float().cpu().numpy(), g0.float().cpu().numpy(), **tol)


def test_noalloc_rejects_rows_beyond_the_scratch():
    from neuratensor_b200 import native
    L = native.load()
    cap = L.nt_noalloc_scratch_bytes()
    dm, di = 1024, 64
    M = cap // (dm * 2) + 1
    x = torch.zeros(1, dm, dtype=torch.bfloat16, device=DEV)   # pointers only; rejected before any launch
    W = torch.zeros(2 * di, dm, dtype=torch.bfloat16, device=DEV)
    out = torch.zeros(1, di, dtype=torch.bfloat16, device=DEV)
    rc = L.nt_rmsnorm_in_proj_noalloc(1, M, dm, di, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                      ctypes.c_void_p(W.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(out.data_ptr()), None)
    assert rc == 1
    assert b"exceeds" in L.nt_last_error()
