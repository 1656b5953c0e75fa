"""Upstream block-scaled GEMMs on tcgen05 (kind::mxf8f6f4) -- drop-in for
docs/reference/kernel.py ``fp8_gemm`` (:277-308) and ``fp4_gemm`` (:562-591).

``C[M, N] = A[M, K] @ B[N, K]^T`` with fp8 e4m3 activations ``a`` and their ue8m0
scales ``a_s`` (as returned by ``act_quant(x, block, scale_fmt="ue8m0",
scale_dtype=torch.float8_e8m0fnu)``), and weights ``b`` in fp8 e4m3 [N, K] with
``b_s`` [ceil(N/block), K/block] (fp8_gemm) or fp4 e2m1 packed [N, K/2] with
``b_s`` [N, K/32] (fp4_gemm).  Only power-of-two (ue8m0) scales are accepted:
the block-scaled MMA multiplies exponents, so upstream's float32 scales have no
form on it.  The output has torch's default dtype unless ``out_dtype`` is given.
"""

from __future__ import annotations

from . import _lib as L


def _u8(t, name):
    v = L.cuda_tensor(t, name)
    return L.u8(v.contiguous())


def _out(a, M, N, out_dtype):
    t = L.torch()
    odt = out_dtype or t.get_default_dtype()
    if odt == t.float32:
        code = L.F32
    elif odt == t.bfloat16:
        code = L.BF16
    else:
        raise ValueError("output dtype must be float32 or bfloat16")
    return t.empty(tuple(a.shape[:-1]) + (N,), dtype=odt, device=a.device), code


def fp8_gemm(a, a_s, b, b_s, scale_dtype=None, block_size: int = 128, out_dtype=None):
    t = L.torch()
    K = a.shape[-1]
    M = a.numel() // K
    N = b.shape[0]
    if a_s.numel() != M * (K // block_size):
        raise ValueError("a_s must hold M * K/block_size scales")
    if tuple(b_s.shape) != ((N + block_size - 1) // block_size, K // block_size):
        raise ValueError("b_s must be [ceil(N/block), K/block]")
    if scale_dtype is not None and scale_dtype == t.float32:
        raise ValueError("only ue8m0 scales are supported by the block-scaled MMA")
    c, code = _out(a, M, N, out_dtype)
    L.call("dsv41_fp8_gemm", L.ptr(_u8(a, "a")), L.ptr(_u8(a_s, "a_s")), L.ptr(_u8(b, "b")),
           L.ptr(_u8(b_s, "b_s")), M, N, K, block_size, L.ptr(c), code, L.stream_of(c))
    return c


def fp4_gemm(a, a_s, b, b_s, scale_dtype=None, act_block_size: int = 128, out_dtype=None):
    t = L.torch()
    K = a.shape[-1]
    M = a.numel() // K
    N = b.shape[0]
    if a_s.numel() != M * (K // act_block_size):
        raise ValueError("a_s must hold M * K/act_block_size scales")
    if tuple(b_s.shape) != (N, K // 32):
        raise ValueError("b_s must be [N, K/32]")
    if scale_dtype is not None and scale_dtype == t.float32:
        raise ValueError("only ue8m0 scales are supported by the block-scaled MMA")
    c, code = _out(a, M, N, out_dtype)
    L.call("dsv41_fp4_gemm", L.ptr(_u8(a, "a")), L.ptr(_u8(a_s, "a_s")), L.ptr(_u8(b, "b")),
           L.ptr(_u8(b_s, "b_s")), M, N, K, act_block_size, L.ptr(c), code, L.stream_of(c))
    return c
