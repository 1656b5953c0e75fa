"""MLX affine quantization on the GPU (mx.quantize as the converter calls it) vs the oracle's
restatement: codes, scales and biases bit-identical.  Parity with MLX itself is unpinned
(MLX is not in the reference tree and no reference test pins its quantizer)."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from oracle import formats as F

pytestmark = pytest.mark.gpu


def _u32(t):
    return t.view(torch.int32).cpu().numpy().view(np.uint32)


def _u16(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _weights(rng, rows, cols, group):
    w = (rng.standard_normal((rows, cols)) * rng.uniform(0.001, 3.0, (rows, 1))).astype(np.float32)
    w[0, :group] = 0.0                                  # all zero
    w[1, :group] = -0.3                                 # constant
    w[2, :group] = np.abs(w[2, :group])                 # one-signed
    w[3, group:2 * group] *= 1000.0                     # large
    return w


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_affine_matches_oracle(cuda, dtype, bits, group):
    rng = np.random.default_rng(bits * 100 + group + (dtype == "bf16"))
    rows, cols = 37, 512
    w = _weights(rng, rows, cols, group)
    if dtype == "bf16":
        w = F.round_bf16(w)
        wt = torch.from_numpy(w).cuda().to(torch.bfloat16)
    else:
        wt = torch.from_numpy(w).cuda()
    wq, s, b = q.dequant.quantize_affine(wt, group, bits)
    owq, os_, ob = F.quantize_affine(w, group, bits, dtype)
    assert wq.shape == (rows, cols * bits // 32) and s.dtype == wt.dtype
    assert np.array_equal(_u32(wq), owq)
    if dtype == "bf16":
        assert np.array_equal(_u16(s), os_) and np.array_equal(_u16(b), ob)
    else:
        assert np.array_equal(s.cpu().numpy().view(np.uint32), os_.view(np.uint32))
        assert np.array_equal(b.cpu().numpy().view(np.uint32), ob.view(np.uint32))
    # the library's own dequantize reads what it wrote as the oracle's dequantize does
    got = q.dequant.dequantize_affine(wq, s, b, group, bits, torch.float32).cpu().numpy()
    want = F.dequant_affine(owq, os_, ob, bits, group, cols, dtype, "f32")
    assert np.array_equal(got, want)


def test_quantize_engram_table_matches_oracle(cuda):
    """convert.quantize_engram_table: fp8 rows + ue8m0 -> fp32 -> bf16 -> affine, in row
    chunks (here 100 rows, so the last chunk is short)."""
    rng = np.random.default_rng(7)
    rows, d, block, bits, group = 250, 256, 32, 4, 64
    wu8 = rng.integers(0, 256, size=(rows, d), dtype=np.uint8)
    wu8[(wu8 & 0x7F) == 0x7F] = 0
    su8 = rng.integers(115, 128, size=(rows, d // block), dtype=np.uint8)
    out = q.convert.quantize_engram_table(torch.from_numpy(wu8).cuda(),
                                          torch.from_numpy(su8).cuda(), bits, group, step=100)
    deq = F.round_bf16(F.dequant_fp8_rows(wu8, su8, block))
    owq, os_, ob = F.quantize_affine(deq, group, bits, "bf16")
    assert np.array_equal(_u32(out["weight"]), owq)
    assert np.array_equal(_u16(out["scales"]), os_) and np.array_equal(_u16(out["biases"]), ob)


def test_release_group_sanitize_and_quantize(cuda, tmp_path):
    """A synthetic release checkpoint through convert.sanitize_group (GPU decode, expert
    stacking) and quantize_tree (experts at 4 bits, the rest at 8): decoded tensors and the
    quantized triples equal the oracle's decode and quantizer."""
    from safetensors.torch import load_file
    import release_fixture as RF
    path, a = RF.write(str(tmp_path / "ckpt"))
    tensors = {}
    for fn in sorted(os.listdir(path)):
        if fn.endswith(".safetensors"):
            tensors.update(load_file(os.path.join(path, fn)))
    out = q.convert.sanitize_group(sorted(tensors), tensors)
    p = a["moe"]
    pre = f"layers.{RF.MOE_LAYER}.ffn"
    for wn, proj in (("w1", "gate_proj"), ("w3", "up_proj"), ("w2", "down_proj")):
        got = out[f"{pre}.experts.{proj}.weight"]
        assert got.dtype == torch.bfloat16 and got.shape[0] == RF.E
        want = np.stack([F.dequant_fp4(p[wn][e], p["s" + wn[1]][e], "bf16") for e in range(RF.E)])
        assert np.array_equal(_u16(got), want)
    got = out[f"{pre}.shared_experts.w1.weight"]
    assert np.array_equal(_u16(got), F.dequant_fp8(p["sw1"], p["ss1"], "bf16"))
    assert out[f"{pre}.gate.bias"].dtype == torch.float32
    assert out[f"layers.{RF.ENGRAM_LAYER}.engram.embed.weight"].dtype == torch.uint8
    qt, modules = q.convert.quantize_tree(out, 8, 4, 64)
    base = f"{pre}.experts.gate_proj"
    assert modules[base] == {"group_size": 64, "bits": 4}
    assert modules[f"{pre}.shared_experts.w1"] == {"group_size": 64, "bits": 8}
    assert f"{pre}.gate" not in modules
    assert f"layers.{RF.ENGRAM_LAYER}.engram.embed" not in modules
    w = F.bf16_bits_to_f32(_u16(out[f"{base}.weight"])).reshape(-1, RF.D)
    owq, os_, ob = F.quantize_affine(w, 64, 4, "bf16")
    assert np.array_equal(_u32(qt[f"{base}.weight"]).reshape(owq.shape), owq)
    assert np.array_equal(_u16(qt[f"{base}.scales"]).reshape(os_.shape), os_)
    assert np.array_equal(_u16(qt[f"{base}.biases"]).reshape(ob.shape), ob)


def test_engram_table_from_checkpoint_matches_in_memory(cuda, tmp_path):
    """The release engram table streamed off disk in row slices (3 slices, the last short)
    converts to the same triple as the table converted in memory."""
    import release_fixture as RF
    path, a = RF.write(str(tmp_path / "ckpt"))
    ckpt = q.release.Checkpoint(path)
    name = f"layers.{RF.ENGRAM_LAYER}.engram.embed.weight"
    got = q.convert.quantize_engram_table_from_checkpoint(ckpt, name, 4, 64, step=400)
    want = q.convert.quantize_engram_table(torch.from_numpy(a["table"]).cuda(),
                                           torch.from_numpy(a["tscale"]).cuda(), 4, 64)
    assert torch.equal(got["weight"].view(torch.int32), want["weight"].view(torch.int32))
    for k in ("scales", "biases"):
        assert torch.equal(got[k], want[k]), k
    assert got["weight"].shape == (RF.ROWS, RF.HD * 4 // 32)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("group,bits", [(32, 2), (64, 4), (128, 8)])
def test_quantize_affine_unaligned_input(cuda, dtype, group, bits):
    """Input not 16-byte aligned (one element past an aligned base): the warp-per-group
    kernel runs instead of the thread-per-group one, with the same bits as the oracle."""
    from deepseek_v41_mlx_b200 import _lib as L
    rng = np.random.default_rng(group + bits)
    rows, cols = 9, 256
    w = _weights(rng, rows, cols, group)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    if dtype == "bf16":
        w = F.round_bf16(w)
    base = torch.zeros(rows * cols + 8, dtype=tdt, device="cuda")
    base[1:1 + rows * cols] = torch.from_numpy(w.reshape(-1)).cuda().to(tdt)
    ptr = base.data_ptr() + base.element_size()               # 2 or 4 bytes past alignment
    wq = torch.empty((rows, cols * bits // 32), dtype=torch.int32, device="cuda")
    s = torch.empty((rows, cols // group), dtype=tdt, device="cuda")
    b = torch.empty_like(s)
    L.call("dsv41_quantize_affine", ptr, L.dtype_code(tdt), rows, cols, group, bits, L.ptr(wq),
           L.ptr(s), L.ptr(b), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    owq, os_, ob = F.quantize_affine(w, group, bits, dtype)
    assert np.array_equal(wq.cpu().numpy().view(np.uint32), owq)
    if dtype == "bf16":
        assert np.array_equal(_u16(s), os_) and np.array_equal(_u16(b), ob)
    else:
        assert np.array_equal(s.cpu().numpy().view(np.uint32), os_.view(np.uint32))
        assert np.array_equal(b.cpu().numpy().view(np.uint32), ob.view(np.uint32))
