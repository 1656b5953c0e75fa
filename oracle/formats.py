"""Weight-format decode, restated in numpy.  Test infrastructure only.

Follows deepseek_v41_mlx/dequant.py:
  e8m0_to_float      dequant.py:33-36   byte b -> 2**(b-127) (fp32; b=255 -> inf as mx.power gives)
  _expand_blocks     dequant.py:39-42   repeat scale grid, crop the ceil overhang
  dequant_fp8        dequant.py:45-50   from_fp8(w) * scale, then cast
  unpack_fp4         dequant.py:53-60   low nibble = even index, LUT _E2M1 (code 8 -> +0.0)
  dequant_fp4        dequant.py:63-68
  dequant_fp8_rows   dequant.py:71-79   row groups of `block` along the last axis, fp32 out
  is_fp4_expert      dequant.py:82-84
The fp4 LUT is the reference's FP4_TABLE (docs/reference/convert.py:13-15).

MLX affine group quantization (not in the reference tree; mlx>=0.32.0, the
layout written at deepseek_v41_mlx/convert.py:156-175 via mx.quantize):
codes are unsigned `bits`-bit integers packed little-endian into uint32 words
(element j of a row at bit offset bits*j of the row's bit stream), one scale
and one bias per `group` consecutive elements.  Oracle definitions (parity
unpinned -- no reference test checks these numerics):
  dequant_affine         out = round_to(out_dtype, fma_f32(scale, q, bias))
  affine_qmm_reference   y = sum_g scale_g * sum_{k in g} x_k q_k + bias_g * sum_{k in g} x_k
                         accumulated in float64 (the mx.quantized_matmul form,
                         which never materialises bf16 weights).
  quantize_affine        mx.quantize as the converter calls it (convert.py:169, :188): per
                         group in fp32, scale = max((max-min)/n, 1e-7) signed toward the
                         larger-magnitude edge, q0 = round(edge/scale), scale = edge/q0 and
                         bias = edge when q0 != 0 (else bias 0), codes = clamp(round((w-bias)
                         /scale), 0, n); rounding half away from zero; scale and bias stored
                         in the input's dtype.  MLX's published scheme as this build restates
                         it -- parity unpinned like the rest of the affine format.
"""

from __future__ import annotations

import numpy as np

FP8_BLOCK = 32
FP4_BLOCK = 32

# e2m1 code -> value; code 8 ("negative zero") maps to +0.0 (dequant.py:29-30).
E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def _e4m3_table() -> np.ndarray:
    """All 256 e4m3fn codes as float32 (bias 7, no inf, NaN at S.1111.111)."""
    t = np.empty(256, dtype=np.float32)
    for b in range(256):
        sign = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = sign * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = sign * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3 = _e4m3_table()


# ---------------------------------------------------------------- bf16 / f16 --

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest-even); returns uint16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = r.astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 -> float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    """Cast float32 to 'f32' (identity), 'bf16' (uint16 bits) or 'f16'."""
    if dtype == "f32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    raise ValueError(dtype)


# ---------------------------------------------------------------- release fp8/fp4 --

def e8m0_to_float(scale_u8: np.ndarray) -> np.ndarray:
    """dequant.py:33-36 -- byte b -> 2**(b-127) in fp32 (0 -> 2^-127, 255 -> inf)."""
    e = np.asarray(scale_u8).astype(np.int32) - 127
    with np.errstate(over="ignore"):
        return np.ldexp(np.float32(1.0), e).astype(np.float32)


def expand_blocks(scale: np.ndarray, rows: int, cols: int, br: int, bc: int) -> np.ndarray:
    """dequant.py:39-42 -- repeat by (br, bc) and crop to [rows, cols]."""
    s = np.repeat(np.repeat(scale, br, axis=0), bc, axis=1)
    return s[:rows, :cols]


def dequant_fp8(weight_u8: np.ndarray, scale_u8: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    """dequant.py:45-50 -- e4m3 [out, in] * ue8m0 [ceil(out/32), ceil(in/32)]."""
    w = E4M3[np.asarray(weight_u8, dtype=np.uint8)]
    rows, cols = w.shape
    s = expand_blocks(e8m0_to_float(scale_u8), rows, cols, FP8_BLOCK, FP8_BLOCK)
    with np.errstate(over="ignore", invalid="ignore"):
        return to_dtype(w * s, dtype)


def unpack_fp4(packed: np.ndarray) -> np.ndarray:
    """dequant.py:53-60 -- [out, in/2] bytes -> f32 [out, in], low nibble first."""
    b = np.asarray(packed).view(np.uint8)
    lo = b & 0x0F
    hi = (b >> 4) & 0x0F
    vals = np.stack([E2M1[lo], E2M1[hi]], axis=-1)
    return vals.reshape(vals.shape[0], -1)


def dequant_fp4(packed: np.ndarray, scale_u8: np.ndarray, dtype: str = "bf16") -> np.ndarray:
    """dequant.py:63-68 -- unpack_fp4 * ue8m0 [out, in/32]."""
    w = unpack_fp4(packed)
    rows, cols = w.shape
    s = expand_blocks(e8m0_to_float(scale_u8), rows, cols, 1, FP4_BLOCK)
    with np.errstate(over="ignore", invalid="ignore"):
        return to_dtype(w * s, dtype)


def dequant_fp8_rows(weight_u8: np.ndarray, scale_u8: np.ndarray, block: int = 32) -> np.ndarray:
    """dequant.py:71-79 -- e4m3 [..., d] * ue8m0 [..., d/block] -> f32."""
    w = E4M3[np.asarray(weight_u8, dtype=np.uint8)]
    s = e8m0_to_float(scale_u8)
    wv = w.reshape(*w.shape[:-1], w.shape[-1] // block, block)
    with np.errstate(over="ignore", invalid="ignore"):
        return (wv * s[..., None]).reshape(w.shape).astype(np.float32)


def is_fp4_expert(name: str) -> bool:
    """dequant.py:82-84."""
    return ".experts." in name and ".shared_experts." not in name


# ---------------------------------------------------------------- MLX affine --

def pack_affine(q: np.ndarray, bits: int) -> np.ndarray:
    """[rows, cols] codes in [0, 2**bits) -> uint32 [rows, cols*bits/32] (LE bit stream)."""
    q = np.asarray(q, dtype=np.uint64)
    rows, cols = q.shape
    if (cols * bits) % 32:
        raise ValueError("cols*bits must be a multiple of 32")
    nw = cols * bits // 32
    out = np.zeros((rows, nw), dtype=np.uint64)
    for j in range(cols):
        bit = bits * j
        w, off = divmod(bit, 32)
        out[:, w] |= (q[:, j] << np.uint64(off)) & np.uint64(0xFFFFFFFF)
        spill = off + bits - 32
        if spill > 0:
            out[:, w + 1] |= q[:, j] >> np.uint64(bits - spill)
    return out.astype(np.uint32)


def unpack_affine(wq: np.ndarray, bits: int, cols: int) -> np.ndarray:
    """Inverse of pack_affine: uint32 [rows, cols*bits/32] -> int codes [rows, cols]."""
    wq = np.asarray(wq, dtype=np.uint32).astype(np.uint64)
    rows = wq.shape[0]
    mask = np.uint64((1 << bits) - 1)
    q = np.empty((rows, cols), dtype=np.int64)
    for j in range(cols):
        bit = bits * j
        w, off = divmod(bit, 32)
        v = wq[:, w] >> np.uint64(off)
        if off + bits > 32:
            v = v | (wq[:, w + 1] << np.uint64(32 - off))
        q[:, j] = (v & mask).astype(np.int64)
    return q


def sb_to_f32(a: np.ndarray, sb_dtype: str) -> np.ndarray:
    if sb_dtype == "bf16":
        return bf16_bits_to_f32(a)
    return np.asarray(a, dtype=np.float32)


def dequant_affine(wq, scales, biases, bits: int, group: int, cols: int,
                   sb_dtype: str = "bf16", out_dtype: str = "bf16") -> np.ndarray:
    """mx.dequantize form: round(out_dtype, fma_f32(s, q, b)).

    fp32 s*q is exact (s has <= 24 significant bits, q <= 8 bits only when s
    is bf16/f16; for f32 scales the fma rounding is reproduced through float64,
    whose product is exact and whose sum is rounded once to float32).
    """
    q = unpack_affine(wq, bits, cols).astype(np.float64)
    s = np.repeat(sb_to_f32(scales, sb_dtype).astype(np.float64), group, axis=1)[:, :cols]
    b = np.repeat(sb_to_f32(biases, sb_dtype).astype(np.float64), group, axis=1)[:, :cols]
    v = (s * q + b).astype(np.float32)   # exact product, sum rounded once to f32
    return to_dtype(v, out_dtype)


def _round_half_away(x: np.ndarray) -> np.ndarray:
    """round() of fp32 values, half away from zero, exact (float64 holds x + 0.5 exactly)."""
    x64 = np.asarray(x, dtype=np.float64)
    return (np.sign(x64) * np.floor(np.abs(x64) + 0.5)).astype(np.float32)


def quantize_affine(w: np.ndarray, group: int, bits: int, sb_dtype: str = "bf16"):
    """mx.quantize(w, group_size=group, bits=bits) as restated in the module docstring:
    fp32 w [rows, cols] -> (uint32 codes [rows, cols*bits/32], scales, biases [rows,
    cols/group] in sb_dtype).  Every step is one IEEE fp32 operation, as the kernel does."""
    w = np.asarray(w, dtype=np.float32)
    rows, cols = w.shape
    g = w.reshape(rows, cols // group, group)
    hi, lo = g.max(-1), g.min(-1)
    nb = np.float32((1 << bits) - 1)
    scale = np.maximum((hi - lo) / nb, np.float32(1e-7)).astype(np.float32)
    side = np.abs(lo) > np.abs(hi)
    scale = np.where(side, scale, -scale).astype(np.float32)
    edge = np.where(side, lo, hi).astype(np.float32)
    q0 = _round_half_away(edge / scale)
    nz = q0 != 0
    scale = np.where(nz, edge / np.where(nz, q0, np.float32(1)), scale).astype(np.float32)
    bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
    q = _round_half_away((g - bias[..., None]) / scale[..., None])
    q = np.clip(q, 0, nb).astype(np.int64).reshape(rows, cols)
    return pack_affine(q, bits), to_dtype(scale, sb_dtype), to_dtype(bias, sb_dtype)


def affine_qmm_reference(x: np.ndarray, wq, scales, biases, bits: int, group: int,
                         sb_dtype: str = "bf16") -> np.ndarray:
    """mx.quantized_matmul form, float64: y[m, n] = sum_k x[m,k] * (s q + b)."""
    x = np.asarray(x, dtype=np.float64)
    cols = x.shape[-1]
    q = unpack_affine(wq, bits, cols).astype(np.float64)
    s = sb_to_f32(scales, sb_dtype).astype(np.float64)
    b = sb_to_f32(biases, sb_dtype).astype(np.float64)
    n, g = s.shape
    xg = x.reshape(x.shape[0], g, group)
    qg = q.reshape(n, g, group)
    acc = np.einsum("mgk,ngk->mng", xg, qg)
    xs = xg.sum(-1)                                  # [m, g]
    return (acc * s[None] + xs[:, None, :] * b[None]).sum(-1)
