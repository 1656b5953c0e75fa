"""Upstream fp8 activation quantization on the GPU.

Same call as docs/reference/kernel.py:98-124 ``act_quant(x, block_size,
scale_fmt, scale_dtype, inplace)``: block-wise e4m3 with the power-of-two
(ue8m0) scale when ``scale_fmt`` is set, or amax/448 otherwise.  Bit-exact with
the reference's CPU transcription tests/kernel_stub.py:47-63.
"""

from __future__ import annotations

from . import _lib as L


def act_quant(x, block_size: int = 128, scale_fmt=None, scale_dtype=None, inplace: bool = False):
    t = L.torch()
    xt = L.cuda_tensor(x, "x")
    if xt.dtype != t.bfloat16:
        raise ValueError("x must be bfloat16")
    if scale_dtype is None:
        scale_dtype = t.float32
    K = xt.shape[-1]
    M = xt.numel() // K if K else 0
    round_scale = 1 if scale_fmt is not None else 0
    q = t.empty(xt.shape, dtype=t.uint8, device=xt.device)
    s_u8 = scale_dtype != t.float32
    s = t.empty(tuple(xt.shape[:-1]) + (K // block_size,), dtype=t.uint8 if s_u8 else t.float32,
                device=xt.device)
    deq = t.empty_like(xt) if inplace else None
    L.call("dsv41_act_quant_fp8", L.ptr(xt), M, K, block_size, round_scale, L.ptr(q), L.ptr(s),
           L.U8 if s_u8 else L.F32, L.ptr(deq) if inplace else None, L.stream_of(xt))
    if inplace:
        x.copy_(deq)
        return x
    qv = q.view(t.float8_e4m3fn)
    if s_u8:
        return qv, s.view(t.float8_e8m0fnu) if scale_dtype == t.float8_e8m0fnu else s
    return qv, s
