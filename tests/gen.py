"""Seeded synthetic inputs with the BASELINE.json value distributions (test helper)."""

from __future__ import annotations

import numpy as np

from oracle import formats as F


def fp8_weight(rng, n, k, scale_lo=118, scale_hi=127):
    """e4m3 bytes uniform over all non-NaN codes; ue8m0 per 32x32 block in [lo, hi]."""
    w = rng.integers(0, 256, size=(n, k), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0
    s = rng.integers(scale_lo, scale_hi + 1, size=((n + 31) // 32, (k + 31) // 32), dtype=np.uint8)
    return w, s


def fp4_weight(rng, n, k, scale_lo=120, scale_hi=128, experts=None):
    """uniform random nibbles packed two per byte; ue8m0 per (row, 32 k) in [lo, hi]."""
    shp = (n, k // 2) if experts is None else (experts, n, k // 2)
    sshp = (n, k // 32) if experts is None else (experts, n, k // 32)
    return (rng.integers(0, 256, size=shp, dtype=np.uint8),
            rng.integers(scale_lo, scale_hi + 1, size=sshp, dtype=np.uint8))


def affine_weight(rng, n, k, bits):
    q = rng.integers(0, 1 << bits, size=(n, k))
    wq = F.pack_affine(q, bits)
    s = F.f32_to_bf16_bits(rng.uniform(0.001, 0.02, size=(n, k // 64)).astype(np.float32))
    b = F.f32_to_bf16_bits((rng.standard_normal((n, k // 64)) * 0.05).astype(np.float32))
    return wq, s, b


def bf16_acts(rng, m, k, std=1.0):
    """N(0, std) rounded to bf16; returns (bf16 bit patterns uint16, float32 values)."""
    b = F.f32_to_bf16_bits((rng.standard_normal((m, k)) * std).astype(np.float32))
    return b, F.bf16_bits_to_f32(b)


def moe_params(rng, E, D, I, with_shared=True):
    p = {}
    gw_b, gw = bf16_acts(rng, E, D, std=D ** -0.5)
    p["gate_w_bits"], p["gate_w"] = gw_b, gw
    p["gate_bias"] = (rng.standard_normal(E) * 0.01).astype(np.float32)
    p["w1"], p["s1"] = fp4_weight(rng, I, D, experts=E)
    p["w3"], p["s3"] = fp4_weight(rng, I, D, experts=E)
    p["w2"], p["s2"] = fp4_weight(rng, D, I, experts=E)
    if with_shared:
        p["sw1"], p["ss1"] = fp8_weight(rng, I, D)
        p["sw3"], p["ss3"] = fp8_weight(rng, I, D)
        p["sw2"], p["ss2"] = fp8_weight(rng, D, I)
    return p
