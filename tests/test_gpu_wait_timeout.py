"""A bounded device wait that runs out, on one GPU, without a fault, trap or hang.

Every device-side wait of the library is bounded by wall time (default 2 s,
``dsv41_set_wait_limit_ns``); when a wait runs out its kernel raises bit 0 of
``dsv41_device_status`` and returns.  Here the wait of the expert-parallel decode
exchange (``k_ep_wait`` through ``dsv41_ep_wait``) is given a flag that nothing
ever publishes: a 2-rank exchange context whose peer does not exist, so rank 1's
step flag stays at zero.  With the limit at 1 ms the kernel must return after about
1 ms, the status bit must be set, and the stream must stay usable.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from deepseek_v41_mlx_b200 import _lib as L
from oracle import formats as F

pytestmark = pytest.mark.gpu


def _status(stream):
    st = C.c_uint32(0)
    L.call("dsv41_device_status", stream, C.byref(st))     # reads and clears
    return st.value


@pytest.mark.parametrize("which", [0, 1])
def test_ep_wait_runs_out_and_reports(cuda, which):
    stream = torch.cuda.current_stream().cuda_stream
    _status(stream)
    ctx = C.c_void_p()
    L.call("dsv41_ep_create", 2, 0, 1, 1, 64, C.byref(ctx))   # never connected: no peer
    try:
        L.call("dsv41_set_wait_limit_ns", 1_000_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        L.call("dsv41_ep_wait", ctx, which, stream)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        assert _status(stream) & 1, "the wait ran out but the status bit is not set"
        assert 0.9 <= ms < 200.0, f"gave up after {ms:.3f} ms (limit 1 ms)"
        # the context and the stream remain usable: a decode kernel gives exact results
        sc = torch.arange(256, dtype=torch.uint8, device="cuda")
        out = torch.empty(256, dtype=torch.float32, device="cuda")
        L.call("dsv41_e8m0_to_float", L.ptr(sc), 256, L.ptr(out), stream)
        want = F.e8m0_to_float(np.arange(256, dtype=np.uint8))
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        assert _status(stream) == 0
    finally:
        L.call("dsv41_set_wait_limit_ns", 0)       # back to the 2 s default
        L.call("dsv41_ep_destroy", ctx)


def test_default_limit_restored_waits_complete(cuda):
    """With the limit back at its default, a pipelined kernel's waits all complete: a GEMV
    over the TMA ring raises no status bit."""
    stream = torch.cuda.current_stream().cuda_stream
    _status(stream)
    rng = np.random.default_rng(1)
    w = torch.from_numpy(rng.integers(0, 256, (512, 1024), dtype=np.uint8)).cuda()
    w[(w & 0x7F) == 0x7F] = 0
    s = torch.from_numpy(rng.integers(118, 128, (16, 32), dtype=np.uint8)).cuda()
    x = torch.randn(4, 1024, device="cuda").to(torch.bfloat16)
    from deepseek_v41_mlx_b200 import linear
    y = linear.linear_fp8(x, w, s, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    assert _status(stream) == 0
