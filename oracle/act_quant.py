"""Upstream fp8 activation quantization, restated in numpy.  Test infrastructure only.

Follows docs/reference/kernel.py:21-37 (fast_log2_ceil / fast_pow2 /
fast_round_scale) and :40-124 (act_quant_kernel), as transcribed by the
reference's own CPU stand-in tests/kernel_stub.py:26-63:
  amax = max(|x| over the block, 1e-4)
  s    = 2**ceil(log2(amax * f32(1/448)))   via IEEE bits      (round_scale)
       = amax / 448                                            (otherwise)
  q    = e4m3_rn(clamp(x / s, -448, 448))
"""

from __future__ import annotations

import numpy as np

from .formats import E4M3

FP8_MAX = 448.0


def pow2_ceil_log2(r: np.ndarray) -> np.ndarray:
    """kernel_stub.py:26-33 -- 2**ceil(log2(r)) via the float32 bit pattern."""
    r = np.ascontiguousarray(r, dtype=np.float32)
    bits = r.view(np.int32)
    exp = ((bits >> 23) & 0xFF) - 127
    man = bits & 0x7FFFFF
    e = exp + (man != 0).astype(np.int32)
    return ((e + 127) << 23).astype(np.int32).view(np.float32)


# all finite, non-negative e4m3 values in increasing order with their codes
_POS_CODES = np.array([c for c in range(0x7F) if not np.isnan(E4M3[c])], dtype=np.uint8)
_POS_VALS = E4M3[_POS_CODES].astype(np.float64)


def f32_to_e4m3(v: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to e4m3fn codes for |v| <= 448 (already clamped)."""
    v = np.asarray(v, dtype=np.float32)
    a = np.abs(v).astype(np.float64)
    i = np.searchsorted(_POS_VALS, a)              # first value >= a
    i = np.clip(i, 1, len(_POS_VALS) - 1)
    lo, hi = _POS_VALS[i - 1], _POS_VALS[i]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (_POS_CODES[i] % 2 == 0))
    code = np.where(pick_hi, _POS_CODES[i], _POS_CODES[i - 1])
    code = np.where(a <= _POS_VALS[0], _POS_CODES[0], code)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    return (code | sign).astype(np.uint8)


def act_quant(x: np.ndarray, block: int = 32, round_scale: bool = True):
    """x f32 [..., K] (values of a bf16 tensor) -> (q codes u8, s f32 [..., K/block])."""
    x = np.asarray(x, dtype=np.float32)
    shp = x.shape
    xb = x.reshape(*shp[:-1], shp[-1] // block, block)
    amax = np.maximum(np.abs(xb).max(-1, keepdims=True), np.float32(1e-4)).astype(np.float32)
    if round_scale:
        s = pow2_ceil_log2(amax * np.float32(1.0 / FP8_MAX))
    else:
        s = (amax / np.float32(FP8_MAX)).astype(np.float32)
    y = np.clip((xb / s).astype(np.float32), -FP8_MAX, FP8_MAX)
    q = f32_to_e4m3(y).reshape(shp)
    return q, s[..., 0]


def act_quant_dequant(x: np.ndarray, block: int = 32, round_scale: bool = True) -> np.ndarray:
    """The inplace=True form: q * s in float32 (caller rounds to its dtype)."""
    q, s = act_quant(x, block, round_scale)
    shp = q.shape
    v = E4M3[q].reshape(*shp[:-1], shp[-1] // block, block) * s[..., None]
    return v.reshape(shp).astype(np.float32)


def s_to_ue8m0(s: np.ndarray) -> np.ndarray:
    """Power-of-two float32 scale -> ue8m0 byte (its biased exponent)."""
    return ((np.ascontiguousarray(s, dtype=np.float32).view(np.int32) >> 23) & 0xFF).astype(np.uint8)
