"""The converter's host rules (convert.py:42-69, :91-153): which tensors are quantized and at
which bits, vision pass-through, orphan scales.  CPU only."""

from __future__ import annotations

import pytest
import torch

import deepseek_v41_mlx_b200 as q


def test_quant_targets_and_bits():
    C = q.convert
    assert C.is_quant_target("layers.3.attn.wq_a.weight", 7168, 64)
    assert C.is_quant_target("layers.3.ffn.experts.down_proj.weight", 2048, 64)
    assert C.is_quant_target("head.weight", 7168, 64)
    assert not C.is_quant_target("layers.3.attn.wo_a.weight", 7168, 64)      # reshaped
    assert not C.is_quant_target("layers.1.engram.embed.weight", 1024, 64)   # stays fp8
    assert not C.is_quant_target("layers.3.attn.compressor.wkv.weight", 7168, 64)
    assert not C.is_quant_target("layers.3.attn.indexer.wk.weight", 7168, 64)
    assert not C.is_quant_target("layers.3.ffn.gate.weight", 7168, 64)        # router
    assert not C.is_quant_target("layers.3.attn.wq_a.weight", 100, 64)       # ragged groups
    assert not C.is_quant_target("layers.3.attn.wq_a.scale", 7168, 64)
    assert C.bits_for("layers.3.ffn.experts.gate_proj.weight", 8, 4) == 4
    assert C.bits_for("layers.3.ffn.shared_experts.w1.weight", 8, 4) == 8
    assert C.bits_for("layers.3.ffn.experts.gate_proj.weight", 8, None) == 8


def test_sanitize_vision_passes_and_orphans_raise():
    C = q.convert
    v = torch.zeros(3)
    out = C.sanitize_group(["vision.patch.weight"], {"vision.patch.weight": v})
    assert out["vision.patch.weight"] is v
    with pytest.raises(ValueError, match="without a weight"):
        C.sanitize_group(["layers.0.attn.wq_a.scale"],
                         {"layers.0.attn.wq_a.scale": torch.zeros(2, dtype=torch.uint8)})
