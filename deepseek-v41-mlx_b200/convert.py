"""The release -> MLX affine conversion steps of deepseek_v41_mlx/convert.py, on the GPU.

The reference's converter dequantizes release tensors and re-quantizes them with
mx.quantize into the mixed 4/8-bit build layout.  Here the decode is the library's
(``dequant``) and the quantizer is ``dequant.quantize_affine`` (MLX's affine scheme as this
library restates it; its numerics are not pinned by a reference test).

    w, s, b = quantize_engram_table(weight_u8, scale_u8, bits=4, group_size=64)
"""

from __future__ import annotations

from . import _lib as L
from . import dequant as D


def quantize_engram_table(weight_u8, scale_u8, bits: int, group_size: int, step: int = 1 << 22):
    """convert.py:178-196: a native fp8 + ue8m0 engram table -> MLX affine triple, in row
    chunks of ``step``: rows dequantized (``dequant_fp8_rows``, fp32), cast to bf16, then
    quantized.  -> {"weight": uint32 codes, "scales": bf16, "biases": bf16}."""
    t = L.torch()
    w = L.u8(L.cuda_tensor(weight_u8, "weight_u8"))
    s = L.u8(L.cuda_tensor(scale_u8, "scale_u8"))
    rows, d = w.shape
    block = d // s.shape[-1]
    out_w = t.empty((rows, d * bits // 32), dtype=t.uint32, device=w.device)
    out_s = t.empty((rows, d // group_size), dtype=t.bfloat16, device=w.device)
    out_b = t.empty_like(out_s)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        deq = D.dequant_fp8_rows(w[r0:r1], s[r0:r1], block).to(t.bfloat16)
        qw, qs, qb = D.quantize_affine(deq, group_size, bits)
        out_w[r0:r1], out_s[r0:r1], out_b[r0:r1] = qw, qs, qb
    return {"weight": out_w, "scales": out_s, "biases": out_b}
