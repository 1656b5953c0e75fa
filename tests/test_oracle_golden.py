"""Pin the CPU oracle against the reference's own outputs (golden fixtures)
and hand-computed known answers.  CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal, golden, rel_fro
from oracle import act_quant as AQ
from oracle import engram as OE
from oracle import formats as F
from oracle import moe as OM


# ---------------------------------------------------------------- formats --

def test_e4m3_table_matches_torch_all_bytes():
    g = golden("dequant_unit_parity.npz")
    assert bits_equal(F.E4M3, g["all_e4m3"])


def test_fp4_table_is_reference_fp4_table():
    g = golden("dequant_unit_parity.npz")
    assert bits_equal(F.E2M1, g["fp4_table"].astype(np.float32))


def test_e2m1_kat_all_nibbles():
    # hand values: 0,.5,1,1.5,2,3,4,6 and their negatives; code 8 is +0.0
    want = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, 0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    packed = np.array([[lo | (hi << 4) for lo, hi in zip(range(0, 16, 2), range(1, 16, 2))]],
                      dtype=np.uint8)
    assert np.array_equal(F.unpack_fp4(packed)[0], np.array(want, np.float32))
    assert not np.signbit(F.unpack_fp4(np.array([[0x08]], np.uint8))[0, 0])


def test_e8m0_kat():
    b = np.array([0, 1, 118, 126, 127, 128, 137, 254, 255], dtype=np.uint8)
    v = F.e8m0_to_float(b)
    assert v[4] == 1.0 and v[3] == 0.5 and v[5] == 2.0 and v[2] == 2.0 ** -9
    assert v[0] == np.float32(2.0 ** -127) and v[7] == np.float32(2.0 ** 127)
    assert np.isinf(v[8])


def test_e4m3_kat():
    # 0x38 = 1.0, 0x7E = 448, 0x01 = 2^-9 (min subnormal), 0xB8 = -1.0, 0x7F = NaN
    assert F.E4M3[0x38] == 1.0 and F.E4M3[0x7E] == 448.0 and F.E4M3[0x01] == 2.0 ** -9
    assert F.E4M3[0xB8] == -1.0 and np.isnan(F.E4M3[0x7F]) and np.isnan(F.E4M3[0xFF])


def test_dequant_unit_parity_golden():
    g = golden("dequant_unit_parity.npz")
    assert bits_equal(F.dequant_fp8(g["wb"], g["sb"], "f32"), g["ref8"])
    assert bits_equal(F.dequant_fp4(g["pb"], g["s4"], "f32"), g["ref4"])
    assert bits_equal(F.dequant_fp8_rows(g["wb"], g["es"], 32), g["refr"])


def test_dequant_fp8_ceil_crop():
    rng = np.random.default_rng(0)
    w = rng.integers(0, 256, size=(70, 45), dtype=np.uint8)
    s = rng.integers(118, 137, size=(3, 2), dtype=np.uint8)
    got = F.dequant_fp8(w, s, "f32")
    for r in (0, 31, 32, 69):
        for c in (0, 31, 32, 44):
            want = F.E4M3[w[r, c]] * 2.0 ** (int(s[r // 32, c // 32]) - 127)
            assert bits_equal(np.float32(want), got[r, c])


def test_bf16_rounding_kat():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -9, -0.0], dtype=np.float32)
    b = F.f32_to_bf16_bits(x)
    assert list(b) == [0x3F80, 0x3F80, 0x3F82, 0x3F80, 0x8000]


def test_affine_pack_roundtrip():
    rng = np.random.default_rng(1)
    for bits in (2, 3, 4, 5, 6, 8):
        q = rng.integers(0, 1 << bits, size=(5, 64), dtype=np.int64)
        assert np.array_equal(F.unpack_affine(F.pack_affine(q, bits), bits, 64), q)
    # 4-bit: element j lives at bits 4*(j%8) of word j//8
    q = np.arange(8, dtype=np.int64)[None] + 1
    assert int(F.pack_affine(q, 4)[0, 0]) == 0x87654321


def test_affine_qmm_matches_dequant_matmul():
    rng = np.random.default_rng(2)
    N, K = 8, 128
    q = rng.integers(0, 16, size=(N, K))
    wq = F.pack_affine(q, 4)
    s = F.f32_to_bf16_bits(rng.uniform(0.001, 0.02, size=(N, K // 64)).astype(np.float32))
    b = F.f32_to_bf16_bits((rng.standard_normal((N, K // 64)) * 0.05).astype(np.float32))
    x = rng.standard_normal((3, K)).astype(np.float32)
    w = F.dequant_affine(wq, s, b, 4, 64, K, "bf16", "f32")
    y = F.affine_qmm_reference(x, wq, s, b, 4, 64)
    assert rel_fro(x.astype(np.float64) @ w.astype(np.float64).T, y) < 1e-6


# ---------------------------------------------------------------- act_quant --

@pytest.mark.parametrize("i", [0, 1, 2])
def test_act_quant_golden(i):
    g = golden("act_quant.npz")
    x = g[f"x{i}"]
    q, s = AQ.act_quant(x, 32, True)
    assert bits_equal(s.reshape(-1), g[f"s{i}"].reshape(-1))
    assert np.array_equal(q, g[f"codes{i}"])
    assert bits_equal(AQ.act_quant_dequant(x, 32, True), g[f"deq{i}"])
    qf, sf = AQ.act_quant(x, 32, False)
    assert bits_equal(sf.reshape(-1), g[f"sf{i}"].reshape(-1))
    assert np.array_equal(qf, g[f"codesf{i}"])


def test_e4m3_rounding_midpoints():
    # midpoint between 1.0 (0x38) and 1.125 (0x39) rounds to even (0x38);
    # midpoint between 1.125 and 1.25 (0x3A) rounds to 0x3A
    v = np.array([1.0625, 1.1875, -1.0625, 2.0 ** -10, 3 * 2.0 ** -10, 448.0], np.float32)
    assert list(AQ.f32_to_e4m3(v)) == [0x38, 0x3A, 0xB8, 0x00, 0x02, 0x7E]


# ---------------------------------------------------------------- engram --

def test_engram_hash_golden():
    g = golden("engram_hash.npz")
    primes, offsets = OE.build_layout(len(g["layer_ids"]), int(g["max_ngram"]), int(g["n_heads"]),
                                      int(g["vocab_size"]))
    assert np.array_equal(primes, g["primes"]) and np.array_equal(offsets, g["offsets"])
    assert tuple(primes.reshape(len(g["layer_ids"]), -1).sum(-1)) == tuple(g["num_embeddings"])
    mult = OE.compute_hash_multipliers(g["layer_ids"], int(g["max_ngram"]),
                                       int(g["token_map_max"]) + 1)
    assert np.array_equal(mult, g["multipliers"])
    # token map restricted to the ids the fixture uses
    tm = np.zeros(int(g["token_map_len"]), dtype=np.int64)
    tm[g["sample_ids"]] = g["token_map_sample"]
    ids, L1 = g["ids"], int(g["L1"])
    cache = np.zeros_like(g["cache"])
    h1 = OE.engram_hash(ids[:, :L1], 0, cache, tm, mult, primes, offsets, int(g["pad_id"]),
                        int(g["max_ngram"]))
    h2 = OE.engram_hash(ids[:, L1:], L1, cache, tm, mult, primes, offsets, int(g["pad_id"]),
                        int(g["max_ngram"]))
    assert np.array_equal(h1, g["h1"]) and np.array_equal(h2, g["h2"])
    assert np.array_equal(cache, g["cache"])


def test_engram_embed_golden():
    g = golden("engram_embed.npz")
    got = OE.gather_rows(g["table"], g["scale"], g["idx"], 32)
    assert bits_equal(got, g["out"])


def test_engram_shard_masking():
    rng = np.random.default_rng(4)
    table = rng.integers(0, 126, size=(40, 64), dtype=np.uint8)
    scale = rng.integers(118, 128, size=(40, 2), dtype=np.uint8)
    idx = rng.integers(0, 40, size=(7, 5))
    full = OE.gather_sum(table, scale, idx, 32, "f32")
    parts = [OE.gather_rows(table[r:r + 10], scale[r:r + 10], idx, 32, row_lo=r)
             for r in range(0, 40, 10)]
    assert np.array_equal(sum(parts), OE.gather_rows(table, scale, idx, 32))
    assert full.shape == (7, 64)


# ---------------------------------------------------------------- router / experts --

def _rx():
    return golden("router_expert.npz")


def test_router_golden():
    g = _rx()
    w, idx, _ = OM.gate(g["x"], g["gate_w"], g["gate_bias"], int(g["topk"]), "sqrtsoftplus",
                        1.0, True, float(g["route_scale"]))
    # same expert sets; weights to fp32 rounding
    assert np.array_equal(np.sort(idx, -1), np.sort(g["indices"], -1))
    order = np.argsort(idx, -1)
    gorder = np.argsort(g["indices"], -1)
    assert np.allclose(np.take_along_axis(w, order, -1),
                       np.take_along_axis(g["weights"], gorder, -1), rtol=2e-6, atol=1e-7)


def test_expert_golden():
    g = _rx()
    e = int(g["e0"])
    y = OM.expert_fp4(g["x"][:5], g["w1"][e], g["s1"][e], g["w3"][e], g["s3"][e], g["w2"][e],
                      g["s2"][e], float(g["swiglu_limit"]), round_bf16_io=False)
    assert rel_fro(y, g["y_expert"]) < 1e-5


def test_moe_layer_golden_exact_mode():
    """Upstream MoE.forward in fp32 (weights before w2) == port order in exact mode."""
    g = _rx()
    p = {k: g[k] for k in ("gate_w", "gate_bias", "w1", "s1", "w3", "s3", "w2", "s2",
                           "sw1", "ss1", "sw3", "ss3", "sw2", "ss2")}
    cfg = dict(topk=int(g["topk"]), score_func="sqrtsoftplus", gate_temp=1.0,
               norm_topk_prob=True, route_scale=float(g["route_scale"]),
               swiglu_limit=float(g["swiglu_limit"]))
    y, _, _ = OM.moe_forward(g["x"], p, cfg, round_bf16_io=False)
    assert rel_fro(y, g["y_moe"]) < 1e-5
    yb, _, _ = OM.moe_forward(g["x"], p, cfg, round_bf16_io=True)
    assert rel_fro(yb, g["y_moe"]) < 1e-2


def test_engram_gate_golden():
    """The gate restatement against upstream Engram.forward (fp32, with and without the
    token mask) on the same kv."""
    g = golden("engram_gate.npz")
    got = OE.engram_gate(g["x"], g["kv"], g["q_weight"], g["k_weight"], float(g["eps"]),
                         float(g["clamp"]))
    np.testing.assert_allclose(got, g["out"], rtol=1e-5, atol=1e-6)
    got = OE.engram_gate(g["x"], g["kv"], g["q_weight"], g["k_weight"], float(g["eps"]),
                         float(g["clamp"]), token_mask=g["mask"])
    np.testing.assert_allclose(got, g["out_masked"], rtol=1e-5, atol=1e-6)
    # kv is the rows' projection
    rows = g["rows"].reshape(g["rows"].shape[:-2] + (-1,))
    np.testing.assert_allclose(rows @ g["wkv"].T, g["kv"], rtol=1e-5, atol=1e-5)
