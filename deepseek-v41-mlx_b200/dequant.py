"""Release-format decode on the GPU -- drop-in for deepseek_v41_mlx/dequant.py.

Same names, arguments and dtype defaults as the reference (dequant.py:24-84);
arrays are torch CUDA tensors (or any DLPack array, converted with
torch.from_dlpack).  Results are bit-exact with the reference's decode: every
value is an fp8/fp4 code times a power-of-two scale.

FP8 e4m3 weights carry one ue8m0 scale per 32x32 block (ceil-cropped at the
edges); FP4 e2m1 experts are packed two per byte with the low nibble at the even
index and one ue8m0 scale per 32 inputs; engram rows carry one ue8m0 scale per
``block`` values.
"""

from __future__ import annotations

from . import _lib as L

FP8_BLOCK = 32
FP4_BLOCK = 32


def _torch():
    return L.torch()


def _out_code(dtype):
    t = _torch()
    if dtype in (t.bfloat16, "bf16", "bfloat16"):
        return t.bfloat16, L.BF16
    if dtype in (t.float32, "f32", "float32"):
        return t.float32, L.F32
    raise ValueError(f"unsupported dtype {dtype!r} (bf16 or float32)")


def e8m0_to_float(scale_u8):
    """dequant.py:33-36 -- byte b -> 2**(b-127) as float32."""
    t = _torch()
    s = L.u8(L.cuda_tensor(scale_u8, "scale_u8"))
    out = t.empty(s.shape, dtype=t.float32, device=s.device)
    L.call("dsv41_e8m0_to_float", L.ptr(s), s.numel(), L.ptr(out), L.stream_of(s))
    return out


def dequant_fp8(weight_u8, scale_u8, dtype=None):
    """dequant.py:45-50 -- e4m3 [out, in] + ue8m0 [ceil(out/32), ceil(in/32)] -> dtype."""
    t = _torch()
    dt, code = _out_code(t.bfloat16 if dtype is None else dtype)
    w = L.u8(L.cuda_tensor(weight_u8, "weight_u8"))
    s = L.u8(L.cuda_tensor(scale_u8, "scale_u8"))
    if w.dim() != 2:
        raise ValueError("weight must be 2-D [out, in]")
    rows, cols = w.shape
    if tuple(s.shape) != ((rows + 31) // 32, (cols + 31) // 32):
        raise ValueError(f"scale shape {tuple(s.shape)} != ceil([{rows}, {cols}] / 32)")
    out = t.empty((rows, cols), dtype=dt, device=w.device)
    L.call("dsv41_dequant_fp8_block", L.ptr(w), L.ptr(s), rows, cols, code, L.ptr(out),
           L.stream_of(w))
    return out


def unpack_fp4(packed):
    """dequant.py:53-60 -- [out, in/2] bytes -> float32 [out, in], low nibble first."""
    t = _torch()
    p = L.u8(L.cuda_tensor(packed, "packed"))
    rows, half = p.shape
    out = t.empty((rows, 2 * half), dtype=t.float32, device=p.device)
    L.call("dsv41_unpack_fp4", L.ptr(p), rows, 2 * half, L.ptr(out), L.stream_of(p))
    return out


def dequant_fp4(packed, scale_u8, dtype=None):
    """dequant.py:63-68 -- packed e2m1 [out, in/2] + ue8m0 [out, in/32] -> dtype."""
    t = _torch()
    dt, code = _out_code(t.bfloat16 if dtype is None else dtype)
    p = L.u8(L.cuda_tensor(packed, "packed"))
    s = L.u8(L.cuda_tensor(scale_u8, "scale_u8"))
    rows, half = p.shape
    cols = 2 * half
    if tuple(s.shape) != (rows, (cols + 31) // 32):
        raise ValueError(f"scale shape {tuple(s.shape)} != [{rows}, ceil({cols}/32)]")
    out = t.empty((rows, cols), dtype=dt, device=p.device)
    L.call("dsv41_dequant_fp4", L.ptr(p), L.ptr(s), rows, cols, code, L.ptr(out), L.stream_of(p))
    return out


def dequant_fp8_rows(weight_u8, scale_u8, block: int = 32):
    """dequant.py:71-79 -- e4m3 [..., d] + ue8m0 [..., d/block] -> float32 [..., d]."""
    t = _torch()
    w = L.u8(L.cuda_tensor(weight_u8, "weight_u8"))
    s = L.u8(L.cuda_tensor(scale_u8, "scale_u8"))
    d = w.shape[-1]
    if d % block or tuple(s.shape) != tuple(w.shape[:-1]) + (d // block,):
        raise ValueError("scale must be [..., d // block]")
    out = t.empty(w.shape, dtype=t.float32, device=w.device)
    rows = w.numel() // d if d else 0
    L.call("dsv41_dequant_fp8_rows", L.ptr(w), L.ptr(s), rows, d, block, L.ptr(out),
           L.stream_of(w))
    return out


def is_fp4_expert(name: str) -> bool:
    """dequant.py:82-84 -- routed-expert matmuls are FP4; shared experts are FP8."""
    return ".experts." in name and ".shared_experts." not in name


def dequantize_affine(wq, scales, biases, group_size: int = 64, bits: int = 4, dtype=None):
    """mx.dequantize for the MLX affine layout (engram.py:219-223): out =
    round(fma_f32(scale, q, bias)); q packed little-endian in uint32 words."""
    t = _torch()
    dt, code = _out_code(t.bfloat16 if dtype is None else dtype)
    w = L.cuda_tensor(wq, "wq")
    if w.dtype not in (t.uint32, t.int32):
        raise ValueError("wq must be uint32 words")
    s = L.cuda_tensor(scales, "scales")
    b = L.cuda_tensor(biases, "biases")
    if s.dtype != b.dtype:
        raise ValueError("scales and biases must share a dtype")
    rows = w.numel() // w.shape[-1]
    cols = w.shape[-1] * 32 // bits
    out = t.empty(tuple(w.shape[:-1]) + (cols,), dtype=dt, device=w.device)
    L.call("dsv41_dequant_affine", L.ptr(w), L.ptr(s), L.ptr(b), L.dtype_code(s.dtype), rows, cols,
           bits, group_size, code, L.ptr(out), L.stream_of(w))
    return out


def quantize_affine(w, group_size: int = 64, bits: int = 4):
    """mx.quantize(w, group_size, bits) for the MLX affine layout, as the converter calls it
    (convert.py:169, :188): w bf16 or fp32 [..., cols] -> (uint32 codes [..., cols*bits/32],
    scales, biases [..., cols/group_size] in w's dtype).  Per group in fp32: the scale spans
    max - min over 2^bits - 1 steps, signed toward the edge of larger magnitude, then set so
    that the edge is a whole number of steps from zero (bias = that edge); codes round half
    away from zero.  group_size 32 / 64 / 128, bits 2 / 4 / 8."""
    t = _torch()
    x = L.cuda_tensor(w, "w")
    if x.dtype not in (t.bfloat16, t.float32):
        x = x.to(t.float32)
    x = x.contiguous()
    cols = x.shape[-1]
    if cols % group_size:
        raise ValueError(f"the last dimension ({cols}) must be a multiple of group_size")
    rows = x.numel() // cols if cols else 0
    lead = tuple(x.shape[:-1])
    wq = t.empty(lead + (cols * bits // 32,), dtype=t.uint32, device=x.device)
    scales = t.empty(lead + (cols // group_size,), dtype=x.dtype, device=x.device)
    biases = t.empty_like(scales)
    L.call("dsv41_quantize_affine", L.ptr(x), L.dtype_code(x.dtype), rows, cols, group_size,
           bits, L.ptr(wq), L.ptr(scales), L.ptr(biases), L.stream_of(x))
    return wq, scales, biases
