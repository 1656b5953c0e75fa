"""The oracle's restatement of mx.quantize (affine group quantization, the converter's step;
parity unpinned: MLX is not in the reference tree and no reference test pins it).  CPU only:
properties of the scheme itself."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import formats as F


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_quantize_affine_properties(bits, group):
    rng = np.random.default_rng(bits * 1000 + group)
    rows, cols = 16, 256
    w = (rng.standard_normal((rows, cols)) * rng.uniform(0.01, 2.0, (rows, 1))).astype(np.float32)
    w[0, :group] = 0.0                                  # an all-zero group
    w[1, :group] = 0.75                                 # a constant group
    w[2, :group] = -np.abs(w[2, :group])                # a one-signed group
    wq, s, b = F.quantize_affine(w, group, bits, "f32")
    n = (1 << bits) - 1
    q = F.unpack_affine(wq, bits, cols)
    assert wq.shape == (rows, cols * bits // 32) and wq.dtype == np.uint32
    assert q.min() >= 0 and q.max() <= n
    sg = np.repeat(s, group, axis=1).astype(np.float64)
    bg = np.repeat(b, group, axis=1).astype(np.float64)
    # elements whose unclamped code lies in [0, n] come back within half a step
    raw = (w.astype(np.float64) - bg) / sg
    inside = (raw >= -0.5) & (raw <= n + 0.5)
    deq = F.dequant_affine(wq, s, b, bits, group, cols, "f32", "f32").astype(np.float64)
    err = np.abs(deq - w)
    assert np.all(err[inside] <= np.abs(sg[inside]) * (0.5 + 1e-5) + 1e-7)
    # zero sits on a code: the bias is 0 or a multiple of the scale apart from it
    z = np.round(-b.astype(np.float64) / s.astype(np.float64))
    resid = np.abs(b.astype(np.float64) + z * s.astype(np.float64))
    assert np.all(resid <= np.abs(b) * 1e-6 + np.abs(s) * 1e-5 + 1e-12)
    # the all-zero group dequantizes to zeros, the constant group to its value
    assert np.all(deq[0, :group] == 0.0)
    assert np.allclose(deq[1, :group], 0.75, rtol=1e-6)


def test_quantize_affine_bf16_scales_are_rounded_fp32():
    rng = np.random.default_rng(3)
    w = rng.standard_normal((4, 128)).astype(np.float32)
    _, s32, b32 = F.quantize_affine(w, 64, 4, "f32")
    wq, s16, b16 = F.quantize_affine(w, 64, 4, "bf16")
    assert np.array_equal(s16, F.f32_to_bf16_bits(s32))
    assert np.array_equal(b16, F.f32_to_bf16_bits(b32))
    assert np.array_equal(wq, F.quantize_affine(w, 64, 4, "f32")[0])


def test_round_half_away():
    x = np.array([0.5, 1.5, 2.5, -0.5, -2.5, 0.49999997, -0.49999997, 0.0], np.float32)
    assert F._round_half_away(x).tolist() == [1, 2, 3, -1, -3, 0, 0, 0]


def _round_div_by_reciprocal(a, s):
    """The kernel's per-element rounding, restated with the same IEEE fp32 steps: y =
    RN(a * RN(1/s)); y's rounding is taken when y is farther than 4e-7|y| + 1e-6 from every
    half-integer, the exact quotient's otherwise.  Returns (result, used_the_product)."""
    a = np.asarray(a, np.float32)
    s = np.asarray(s, np.float32)
    rs = np.float32(1.0) / s
    y = (a * rs).astype(np.float32)
    d = np.abs((y - np.floor(y)).astype(np.float32) - np.float32(0.5)).astype(np.float32)
    m = (np.abs(y).astype(np.float64) * np.float64(np.float32(4e-7))
         + np.float64(np.float32(1e-6))).astype(np.float32)
    fast = d > m
    exact = F._round_half_away((a / s).astype(np.float32))
    return np.where(fast, F._round_half_away(y), exact), fast


def test_reciprocal_rounding_matches_the_divide():
    """Random operands and adversarial ones a few ulps from (k + 0.5) * s: the product's
    rounding, where the margin lets it stand, equals the correctly rounded quotient's."""
    rng = np.random.default_rng(11)
    s = rng.uniform(1e-4, 3.0, 200000).astype(np.float32) * rng.choice([-1, 1], 200000)
    a = (rng.uniform(-300, 300, 200000).astype(np.float32) * np.abs(s)).astype(np.float32)
    k = rng.integers(-260, 260, 200000).astype(np.float32)
    tie = ((k + np.float32(0.5)) * s).astype(np.float32)
    for ulps in (-3, -1, 0, 1, 3):
        adv = np.nextafter(tie, np.float32(np.inf) if ulps > 0 else np.float32(-np.inf)) \
            if ulps else tie
        for _ in range(abs(ulps) - 1 if ulps else 0):
            adv = np.nextafter(adv, np.float32(np.inf) if ulps > 0 else np.float32(-np.inf))
        a = np.concatenate([a, adv.astype(np.float32)])
    s_all = np.resize(s, a.shape)
    got, fast = _round_div_by_reciprocal(a, s_all)
    want = F._round_half_away((a / s_all).astype(np.float32))
    assert np.array_equal(got, want)
    assert fast[:200000].mean() > 0.9             # random operands: the divide is rare
    near = np.abs((a / s_all) - np.floor(a / s_all) - 0.5) < 1e-7
    assert not fast[near].any()
