"""The release -> MLX affine conversion steps of deepseek_v41_mlx/convert.py, on the GPU.

The reference's converter dequantizes release tensors and re-quantizes them with
mx.quantize into the mixed 4/8-bit build layout.  Here the decode is the library's
(``dequant``) and the quantizer is ``dequant.quantize_affine`` (MLX's affine scheme as this
library restates it; its numerics are not pinned by a reference test).

    w, s, b = quantize_engram_table(weight_u8, scale_u8, bits=4, group_size=64)
"""

from __future__ import annotations

import re

from . import _lib as L
from . import dequant as D

# tensors passed through untouched (convert.py:42)
VISION_PREFIXES = ("vision.", "aligner.", "image_start", "image_end", "image_newline")
# kept unquantized whatever the shapes (convert.py:44-51): wo_a is reshaped block-diagonally
# by attention (a packed weight would be carved as bytes), the engram table stays native fp8,
# the compressor and the indexer's wk / weights_proj are small and precision-sensitive
_NEVER_QUANT = re.compile(
    r"(\.wo_a\.|\.engram\.embed\.|\.compressor\.|\.indexer\.wk\.|\.weights_proj\.)")
_QUANTIZABLE = ("wq_a", "wq_b", "wkv", "wo_b", "w1", "w2", "w3", "gate_proj", "up_proj",
                "down_proj", "embed", "head")
_EXPERT = re.compile(r"(layers\.\d+\.ffn\.experts)\.(\d+)\.(w[123])\.weight$")
_KEEP_F32 = re.compile(r"(hc_\w+|attn_sink|gate\.bias(_vl)?)$")


def is_quant_target(name: str, in_dim: int, group_size: int) -> bool:
    """convert.py:53-63: a ``.weight`` of one of the quantizable projections whose input
    dimension is a whole number of groups, and not one of the kept modules."""
    if not name.endswith(".weight") or _NEVER_QUANT.search(name) or in_dim % group_size:
        return False
    parts = name.rsplit(".", 2)
    return len(parts) >= 2 and parts[-2] in _QUANTIZABLE


def bits_for(name: str, bits: int, expert_bits: int | None) -> int:
    """convert.py:66-69: routed experts at ``expert_bits`` when given, all else at ``bits``."""
    return expert_bits if expert_bits and D.is_fp4_expert(name) else bits


def sanitize_group(names, tensors, dtype=None):
    """convert.py:91-153 on the GPU: one group of release tensors (torch, any device) -> final
    name -> CUDA tensor.
    fp8 (32x32 ue8m0) and fp4 (routed experts) weights are decoded to ``dtype`` (bf16) by the
    library's kernels; routed experts are stacked into ``*.{gate,up,down}_proj.weight``
    [E, out, in]; the engram table and its scales stay native (uint8); hc_* / attn_sink /
    gate.bias(_vl) become fp32; vision tensors pass through.  A scale with no weight raises
    ValueError, as the reference does."""
    t = L.torch()
    dtype = dtype or t.bfloat16
    out, consumed, experts = {}, set(), {}
    for name in names:
        if name in consumed:
            continue
        if name.startswith(VISION_PREFIXES):
            out[name] = tensors[name]
            continue
        if name.endswith(".scale"):
            continue                                     # taken with its weight
        w = tensors[name].cuda()
        if ".engram.embed." in name:
            sname = name[:-len(".weight")] + ".scale"
            out[name] = L.u8(w)
            out[sname] = L.u8(tensors[sname].cuda())
            consumed.add(sname)
            continue
        sname = name[:-len(".weight")] + ".scale" if name.endswith(".weight") else None
        if sname is not None and sname in tensors:
            consumed.add(sname)
            s = L.u8(tensors[sname].cuda())
            w = (D.dequant_fp4(w, s, dtype) if D.is_fp4_expert(name)
                 else D.dequant_fp8(L.u8(w), s, dtype))
        m = _EXPERT.match(name)
        if m:
            proj = {"w1": "gate_proj", "w3": "up_proj", "w2": "down_proj"}[m.group(3)]
            experts.setdefault(f"{m.group(1)}.{proj}.weight", {})[int(m.group(2))] = w
            continue
        if _KEEP_F32.search(name):
            w = w.float()
        out[name] = w
    for final, parts in experts.items():
        n = len(parts)
        if sorted(parts) != list(range(n)):
            raise ValueError(f"missing experts for {final}")
        out[final] = t.stack([parts[i] for i in range(n)])
    orphans = [n for n in names if n.endswith(".scale") and n not in consumed
               and not n.startswith(VISION_PREFIXES)]
    if orphans:
        raise ValueError(f"{len(orphans)} scale tensors without a weight, "
                         f"e.g. {orphans[:3]} -- layout change?")
    return out


def quantize_tree(weights, bits: int, expert_bits: int | None, group_size: int):
    """convert.py:156-175 on the GPU: every eligible ``.weight`` replaced by the MLX affine
    triple ``.weight`` (uint32 codes) / ``.scales`` / ``.biases`` (``dequant.quantize_affine``),
    plus {module path: {"group_size", "bits"}} for the loader to replay."""
    out, modules = {}, {}
    for name, w in weights.items():
        if name.startswith(VISION_PREFIXES) or not is_quant_target(name, w.shape[-1], group_size):
            out[name] = w
            continue
        b = bits_for(name, bits, expert_bits)
        wq, sc, bi = D.quantize_affine(w, group_size, b)
        base = name[:-len(".weight")]
        out[f"{base}.weight"], out[f"{base}.scales"], out[f"{base}.biases"] = wq, sc, bi
        modules[base] = {"group_size": group_size, "bits": b}
    return out, modules


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


def quantize_engram_table_from_checkpoint(ckpt, weight_name: str, bits: int, group_size: int,
                                          step: int = 1 << 22):
    """convert.py:199-226: a release engram table streamed off disk in row slices (never the
    whole 98 GB tensor in host memory) into the MLX affine triple, on the GPU.  ``ckpt`` is a
    ``release.Checkpoint``; ``weight_name`` the table's ``.weight`` (its ``.scale`` beside
    it).  The same chunk arithmetic as ``quantize_engram_table`` (quantization is row-local),
    so the result is identical to converting the table in one piece."""
    t = L.torch()
    sname = weight_name[:-len(".weight")] + ".scale"
    rows, d = ckpt.shape(weight_name)
    block = d // ckpt.shape(sname)[-1]
    out_w = t.empty((rows, d * bits // 32), dtype=t.uint32, device="cuda")
    out_s = t.empty((rows, d // group_size), dtype=t.bfloat16, device="cuda")
    out_b = t.empty_like(out_s)
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        w = ckpt.get(weight_name, "cuda", rows=(r0, r1))
        s = ckpt.get(sname, "cuda", rows=(r0, r1))
        deq = D.dequant_fp8_rows(w, s, block).to(t.bfloat16)
        out_w[r0:r1], out_s[r0:r1], out_b[r0:r1] = D.quantize_affine(deq, group_size, bits)
    return {"weight": out_w, "scales": out_s, "biases": out_b}
