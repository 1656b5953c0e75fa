"""The allocation-free fp8 GEMV entry point (dsv41_gemv_fp8_block_noalloc).

It exists for callers that cannot give the library device memory: hosts that own
all GPU memory through their own pool, and FFI callers without a device
allocator.  Its output must match the workspace entry point
(dsv41_gemv_fp8_block) within the GEMV tolerance used elsewhere (1e-5 relative
Frobenius, fp32 output), on two calls in a row (the shared scratch array keeps
the previous call's contents).  This file is collected last on purpose.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import rel_fro
from deepseek_v41_mlx_b200 import _lib as L
from gen import bf16_acts, fp8_weight

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


_DT = {L.F32: torch.float32, L.BF16: torch.bfloat16}


def _gemv_workspace(lib, x, w, s, M, K, N, stream, odt=L.F32):
    y = torch.empty((M, N), dtype=_DT[odt], device="cuda")
    ws = torch.empty(lib.dsv41_gemv_workspace_size(M, N, K), dtype=torch.uint8, device="cuda")
    st = lib.dsv41_gemv_fp8_block(x.data_ptr(), M, K, w.data_ptr(), s.data_ptr(), N, odt,
                                  y.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    assert st == 0, L.last_error()
    return y


def _gemv_noalloc(lib, x, w, s, M, K, N, stream, odt=L.F32):
    y = torch.empty((M, N), dtype=_DT[odt], device="cuda")
    st = lib.dsv41_gemv_fp8_block_noalloc(x.data_ptr(), M, K, w.data_ptr(), s.data_ptr(), N, odt,
                                          y.data_ptr(), stream)
    assert st == 0, L.last_error()
    return y


# (M, N, K, output): every activation-tile width (M <= 8, <= 16, <= 32), bf16 output, and
# a shape whose split-K count the 4 MiB array caps below the workspace entry point's
@pytest.mark.parametrize("M,N,K,odt", [(1, 4096, 7168, L.F32), (32, 512, 2048, L.F32),
                                       (5, 200, 1024, L.F32), (12, 4096, 7168, L.F32),
                                       (12, 4096, 7168, L.BF16), (32, 16384, 8192, L.F32)])
def test_noalloc_matches_workspace_entry_point(cuda, M, N, K, odt):
    lib = L.load()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(M + N + K)
    w, s = fp8_weight(rng, N, K)
    wd, sd = _d(w), _d(s)
    tol = 1e-5 if odt == L.F32 else 1e-2       # fp32 / bf16 output, as the other GEMV tests
    for call in range(2):                       # two calls in a row share the scratch
        xb, _ = bf16_acts(rng, M, K)
        x = _d(xb.view(np.int16)).view(torch.bfloat16)
        ref = _gemv_workspace(lib, x, wd, sd, M, K, N, stream, odt)
        got = _gemv_noalloc(lib, x, wd, sd, M, K, N, stream, odt)
        torch.cuda.synchronize()
        assert rel_fro(got.float().cpu().numpy(), ref.float().cpu().numpy()) < tol, f"call {call}"


def test_noalloc_rejects_oversized_shapes(cuda):
    lib = L.load()
    st = lib.dsv41_gemv_fp8_block_noalloc(None, 33, 1024, None, None, 64, L.F32, None, None)
    assert st == L.UNSUPPORTED and "workspace" in L.last_error()
    st = lib.dsv41_gemv_fp8_block_noalloc(None, 32, 16384, None, None, 64, L.F32, None, None)
    assert st == L.UNSUPPORTED
    st = lib.dsv41_gemv_fp8_block_noalloc(None, 1, 1024, None, None, 16385, L.F32, None, None)
    assert st == L.UNSUPPORTED
    # empty shapes are a no-op, as for dsv41_gemv_fp8_block
    assert lib.dsv41_gemv_fp8_block_noalloc(None, 0, 1024, None, None, 64, L.F32, None, None) == 0
    assert lib.dsv41_gemv_fp8_block_noalloc(None, 3, 1024, None, None, 0, L.F32, None, None) == 0
    flags = C.c_uint32(0)
    L.call("dsv41_device_status", torch.cuda.current_stream().cuda_stream, C.byref(flags))
    assert flags.value == 0
