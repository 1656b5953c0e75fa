"""Dequant-then-matmul products, restated in numpy.  Test infrastructure only.

The a16 form of upstream ``linear()`` (docs/reference/model.py:181-207) as the
MLX port runs it after conversion: weights decoded exactly (dequant.py:45-68)
and multiplied by the un-quantized activations (deepseek_v41_mlx/convert.py:
119-127 + nn.Linear).  Accumulation is float64 so the oracle is tighter than
any fp32 kernel; outputs are float32 unless noted.

The a8 form (upstream fp8_gemm / fp4_gemm, docs/reference/kernel.py:207-307,
:477-591): activations go through act_quant first and the per-32 activation
scale and weight scale are applied per K block; since every scale is a power
of two the product equals dequant(a) . dequant(w)^T exactly, which is what is
computed here.
"""

from __future__ import annotations

import numpy as np

from . import act_quant as AQ
from .formats import (E4M3, affine_qmm_reference, bf16_bits_to_f32, dequant_affine,
                      dequant_fp4, dequant_fp8)


def _mm(x: np.ndarray, w: np.ndarray, acc=np.float64) -> np.ndarray:
    return (np.asarray(x, dtype=acc) @ np.asarray(w, dtype=acc).T).astype(np.float32)


def linear_fp8_block(x, w_u8, s_u8, acc=np.float64):
    """y = x . dequant_fp8(w)^T  (x float32 values of bf16 activations)."""
    return _mm(x, dequant_fp8(w_u8, s_u8, "f32"), acc)


def linear_fp4(x, w_packed, s_u8, acc=np.float64):
    """y = x . dequant_fp4(w)^T."""
    return _mm(x, dequant_fp4(w_packed, s_u8, "f32"), acc)


def linear_affine(x, wq, scales, biases, bits, group=64, sb_dtype="bf16"):
    """mx.quantized_matmul form (see formats.affine_qmm_reference)."""
    return affine_qmm_reference(x, wq, scales, biases, bits, group, sb_dtype).astype(np.float32)


def linear_affine_bf16w(x, wq, scales, biases, bits, group=64):
    """The quantized matmul with the weights dequantized to bf16 first (mx.dequantize,
    then a bf16 matmul -- the form MLX's quantized matmul evaluates for bf16 inputs),
    float64 accumulation, float32 out."""
    w = bf16_bits_to_f32(dequant_affine(wq, scales, biases, bits, group, np.asarray(x).shape[-1]))
    return _mm(x, w)


def act_dequant(x, block=32):
    """Upstream act_quant(x, 32, 'ue8m0') followed by exact decode (a8 activations)."""
    q, s = AQ.act_quant(x, block, True)
    shp = q.shape
    v = E4M3[q].reshape(*shp[:-1], shp[-1] // block, block) * s[..., None]
    return v.reshape(shp).astype(np.float32)


def linear_fp4_a8(x, w_packed, s_u8):
    """Upstream fp4_gemm(act_quant(x)) in exact arithmetic, float32 out."""
    return _mm(act_dequant(x), dequant_fp4(w_packed, s_u8, "f32"))


def linear_fp8_block_a8(x, w_u8, s_u8):
    """Upstream fp8_gemm(act_quant(x)) in exact arithmetic, float32 out."""
    return _mm(act_dequant(x), dequant_fp8(w_u8, s_u8, "f32"))
