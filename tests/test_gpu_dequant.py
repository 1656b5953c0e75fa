"""GPU decode kernels vs the oracle and the reference's golden vectors: bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import bits_equal, golden
from oracle import formats as F

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bf16_bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def test_golden_dequant_unit_parity(cuda):
    g = golden("dequant_unit_parity.npz")
    D = q.dequant
    assert bits_equal(D.dequant_fp8(_d(g["wb"]), _d(g["sb"]), torch.float32).cpu().numpy(), g["ref8"])
    assert bits_equal(D.dequant_fp4(_d(g["pb"]), _d(g["s4"]), torch.float32).cpu().numpy(), g["ref4"])
    assert bits_equal(D.dequant_fp8_rows(_d(g["wb"]), _d(g["es"])).cpu().numpy(), g["refr"])


def test_e8m0_all_bytes(cuda):
    b = np.arange(256, dtype=np.uint8)
    got = q.dequant.e8m0_to_float(_d(b)).cpu().numpy()
    assert bits_equal(got, F.e8m0_to_float(b))


@pytest.mark.parametrize("shape", [(96, 64), (70, 45), (33, 8), (1, 1)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_dequant_fp8_all_codes(cuda, shape, dtype):
    rng = np.random.default_rng(sum(shape))
    w = rng.integers(0, 256, size=shape, dtype=np.uint8)          # includes NaN codes
    s = rng.integers(0, 256, size=((shape[0] + 31) // 32, (shape[1] + 31) // 32), dtype=np.uint8)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    got = q.dequant.dequant_fp8(_d(w), _d(s), tdt)
    want = F.dequant_fp8(w, s, dtype)
    got = got.cpu().numpy() if dtype == "f32" else _bf16_bits(got)
    if dtype == "bf16":   # NaN payloads may differ; compare NaN-ness then the rest
        nan = (want & 0x7FFF) > 0x7F80
        assert np.array_equal(nan, (got & 0x7FFF) > 0x7F80)
        assert np.array_equal(np.where(nan, 0, got), np.where(nan, 0, want))
    else:
        assert bits_equal(got, want)


@pytest.mark.parametrize("shape", [(96, 64), (5, 30), (64, 2)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_dequant_fp4(cuda, shape, dtype):
    rng = np.random.default_rng(shape[0])
    p = rng.integers(0, 256, size=(shape[0], shape[1] // 2), dtype=np.uint8)
    s = rng.integers(100, 150, size=(shape[0], (shape[1] + 31) // 32), dtype=np.uint8)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    got = q.dequant.dequant_fp4(_d(p), _d(s), tdt)
    got = got.cpu().numpy() if dtype == "f32" else _bf16_bits(got)
    assert bits_equal(got, F.dequant_fp4(p, s, dtype))


def test_unpack_fp4_all_nibbles(cuda):
    p = np.arange(256, dtype=np.uint8).reshape(4, 64)
    got = q.dequant.unpack_fp4(_d(p)).cpu().numpy()
    assert bits_equal(got, F.unpack_fp4(p))          # includes code 8 -> +0.0


@pytest.mark.parametrize("block", [32, 256, 1024])
def test_dequant_fp8_rows(cuda, block):
    rng = np.random.default_rng(block)
    w = rng.integers(0, 256, size=(7, 3, 1024), dtype=np.uint8)
    s = rng.integers(110, 140, size=(7, 3, 1024 // block), dtype=np.uint8)
    got = q.dequant.dequant_fp8_rows(_d(w), _d(s), block).cpu().numpy()
    assert bits_equal(got, F.dequant_fp8_rows(w, s, block))


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
@pytest.mark.parametrize("sb", ["bf16", "f16", "f32"])
def test_dequant_affine(cuda, bits, sb):
    rng = np.random.default_rng(bits)
    rows, cols, group = 9, 256, 64
    qv = rng.integers(0, 1 << bits, size=(rows, cols))
    wq = F.pack_affine(qv, bits)
    sf = rng.uniform(0.001, 0.02, size=(rows, cols // group)).astype(np.float32)
    bf = (rng.standard_normal((rows, cols // group)) * 0.05).astype(np.float32)
    if sb == "bf16":
        s, b = F.f32_to_bf16_bits(sf), F.f32_to_bf16_bits(bf)
        ts, tb = _d(s.view(np.int16)).view(torch.bfloat16), _d(b.view(np.int16)).view(torch.bfloat16)
    elif sb == "f16":
        s, b = sf.astype(np.float16), bf.astype(np.float16)
        ts, tb = _d(s), _d(b)
    else:
        s, b = sf, bf
        ts, tb = _d(s), _d(b)
    got = q.dequant.dequantize_affine(_d(wq.view(np.int32)), ts, tb, group, bits, torch.float32)
    want = F.dequant_affine(wq, s, b, bits, group, cols, sb, "f32")
    assert bits_equal(got.cpu().numpy(), want)
    gotb = q.dequant.dequantize_affine(_d(wq.view(np.int32)), ts, tb, group, bits, torch.bfloat16)
    assert np.array_equal(_bf16_bits(gotb), F.dequant_affine(wq, s, b, bits, group, cols, sb, "bf16"))


def test_dequant_fp8_baseline_shape(cuda):
    """config 1 weight [4096, 7168]: bf16 output equals the exact f32 output rounded."""
    g = torch.Generator(device="cuda").manual_seed(0)
    w = torch.randint(0, 256, (4096, 7168), dtype=torch.uint8, device="cuda", generator=g)
    w[(w & 0x7F) == 0x7F] = 0
    s = torch.randint(118, 128, (128, 224), dtype=torch.uint8, device="cuda", generator=g)
    f = q.dequant.dequant_fp8(w, s, torch.float32)
    b = q.dequant.dequant_fp8(w, s, torch.bfloat16)
    assert torch.equal(f.to(torch.bfloat16), b)
    rows = np.array([0, 31, 32, 4095])
    # each sampled row with its own 32-row scale block
    want = np.stack([F.dequant_fp8(w[r:r + 1].cpu().numpy(), s[r // 32:r // 32 + 1].cpu().numpy(),
                                   "f32")[0] for r in rows])
    assert bits_equal(f[rows].cpu().numpy(), want)
