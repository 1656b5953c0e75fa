"""Engram hash and row gather vs the reference goldens and the oracle: bit-exact."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import bits_equal, golden, rel_fro
from oracle import engram as OE

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _args_from_golden(g):
    return types.SimpleNamespace(
        engram_layer_ids=tuple(int(v) for v in g["layer_ids"]),
        engram_num_embeddings=tuple(int(v) for v in g["num_embeddings"]),
        engram_max_ngram_size=int(g["max_ngram"]), engram_vocab_size=int(g["vocab_size"]),
        engram_n_heads=int(g["n_heads"]), engram_pad_id=2,
        engram_compressed_vocab_size=int(g["token_map_max"]) + 1)


def _token_map(g):
    """The real map restricted to the ids the fixture uses, plus one unused id that
    carries the largest compressed id (the compressed-vocab size check)."""
    tm = np.zeros(int(g["token_map_len"]), dtype=np.int64)
    tm[g["sample_ids"]] = g["token_map_sample"]
    spare = np.setdiff1d(np.arange(len(tm)), g["sample_ids"])[0]
    tm[spare] = int(g["token_map_max"])
    return tm


def test_hash_golden_release_config(cuda):
    """Release layout (layers 1 and 14, 16M vocab, 8 heads) and the real token map,
    two chunks through one id cache."""
    g = golden("engram_hash.npz")
    tm = _token_map(g)
    args = _args_from_golden(g)
    h = q.engram.EngramHasher(args, tm)
    cache = torch.zeros(g["cache"].shape, dtype=torch.int64, device="cuda")
    ids, L1 = g["ids"], int(g["L1"])
    h1 = h(_d(ids[:, :L1]), 0, cache)
    h2 = h(_d(ids[:, L1:]), L1, cache)
    assert np.array_equal(h1.cpu().numpy(), g["h1"])
    assert np.array_equal(h2.cpu().numpy(), g["h2"])
    assert np.array_equal(cache.cpu().numpy(), g["cache"])


def test_hash_numpy_cache_written_back(cuda):
    g = golden("engram_hash.npz")
    tm = _token_map(g)
    h = q.engram.EngramHasher(_args_from_golden(g), tm)
    cache = np.zeros_like(g["cache"])
    ids, L1 = g["ids"], int(g["L1"])
    h(ids[:, :L1], 0, cache)
    assert np.array_equal(cache[:, :L1], g["cache"][:, :L1])


def test_hash_baseline_layout(cuda):
    """config 5 layout: one layer, 24 primes from 4,000,000 (about 96M rows)."""
    rng = np.random.default_rng(5)
    primes, offsets = OE.build_layout(1, 4, 8, 4_000_000)
    mult = OE.compute_hash_multipliers((1,), 4, 99092)
    tm = np.arange(99092, dtype=np.int64)
    args = types.SimpleNamespace(engram_layer_ids=(1,), engram_num_embeddings=(int(primes.sum()),),
                                 engram_max_ngram_size=4, engram_vocab_size=4_000_000,
                                 engram_n_heads=8, engram_pad_id=2,
                                 engram_compressed_vocab_size=99092)
    h = q.engram.EngramHasher(args, tm)
    ids = rng.integers(0, 99092, size=(2, 700), dtype=np.int64)
    cache = torch.zeros((2, 1024), dtype=torch.int64, device="cuda")
    got = h(_d(ids), 0, cache).cpu().numpy()
    cache_np = np.zeros((2, 1024), dtype=np.int64)
    want = OE.engram_hash(ids, 0, cache_np, tm, mult, primes, offsets, 2, 4)
    assert np.array_equal(got, want)
    assert got.min() >= 0 and got.max() < primes.sum()


def test_gather_rows_golden(cuda):
    g = golden("engram_embed.npz")
    emb = q.engram.EngramEmbedding(g["table"].shape[0], g["table"].shape[1], 32)
    emb.weight, emb.scale = _d(g["table"]), _d(g["scale"])
    got = emb(_d(g["idx"])).cpu().numpy()
    assert bits_equal(got, g["out"])


# T=400: more tokens than the GPU holds warps at once
@pytest.mark.parametrize("d,block", [(256, 32), (1024, 1024), (512, 64), (1024, 32)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("T", [29, 400])
def test_gather_sum_every_scale_and_code(cuda, d, block, dtype, T):
    """Every ue8m0 byte (0 .. 255: subnormal to infinite scales, where products overflow) and
    every e4m3 code (NaN included), plain and packed rows: the bits of the oracle's rounded
    product then rounded sum, NaN for NaN."""
    rng = np.random.default_rng(7 * d + block + T)
    rows = 3000
    table = rng.integers(0, 256, size=(rows, d), dtype=np.uint8)
    scale = rng.integers(0, 256, size=(rows, d // block), dtype=np.uint8)
    idx = rng.integers(0, rows, size=(T, 24))
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    want = OE.gather_sum(table, scale, idx, block, dtype)
    for packed in (False, True):
        emb = q.engram.EngramEmbedding(rows, d, block)
        emb.weight, emb.scale = _d(table), _d(scale)
        if packed:
            emb.pack()
        got = emb.gather_sum(_d(idx), tdt)
        got = got.cpu().numpy() if dtype == "f32" else got.view(torch.int16).cpu().numpy().view(np.uint16)
        if dtype == "bf16":              # any NaN pattern is NaN
            nan_w = (want & 0x7F80) == 0x7F80
            nan_w &= (want & 0x7F) != 0
            nan_g = ((got & 0x7F80) == 0x7F80) & ((got & 0x7F) != 0)
            assert np.array_equal(nan_w, nan_g), packed
            assert np.array_equal(np.where(nan_w, 0, want), np.where(nan_g, 0, got)), packed
        else:
            assert bits_equal(got, want), packed


@pytest.mark.parametrize("d,block", [(256, 32), (1024, 1024), (512, 64)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_gather_sum(cuda, d, block, dtype):
    rng = np.random.default_rng(d + block)
    rows = 5000
    table = rng.integers(0, 256, size=(rows, d), dtype=np.uint8)
    table[(table & 0x7F) == 0x7F] = 0
    scale = rng.integers(115, 128, size=(rows, d // block), dtype=np.uint8)
    idx = rng.integers(0, rows, size=(37, 24))
    emb = q.engram.EngramEmbedding(rows, d, block)
    emb.weight, emb.scale = _d(table), _d(scale)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    got = emb.gather_sum(_d(idx), tdt)
    want = OE.gather_sum(table, scale, idx, block, dtype)
    got = got.cpu().numpy() if dtype == "f32" else got.view(torch.int16).cpu().numpy().view(np.uint16)
    assert bits_equal(got, want)


def test_gather_sharded_sums_to_full(cuda):
    """row-sharded lookups (ids off the shard read zero rows) add up to the full lookup."""
    rng = np.random.default_rng(8)
    rows, d, block, ws = 4000, 256, 32, 4
    table = rng.integers(0, 126, size=(rows, d), dtype=np.uint8)
    scale = rng.integers(115, 128, size=(rows, d // block), dtype=np.uint8)
    idx = _d(rng.integers(0, rows, size=(9, 24)))
    full = q.engram.EngramEmbedding(rows, d, block)
    full.weight, full.scale = _d(table), _d(scale)
    ref = full(idx)
    part = (rows + ws - 1) // ws
    acc = torch.zeros_like(ref)
    for r in range(ws):
        e = q.engram.EngramEmbedding(part, d, block, row_lo=r * part)
        e.weight, e.scale = _d(table[r * part:(r + 1) * part]), _d(scale[r * part:(r + 1) * part])
        acc += e(idx)
    assert torch.equal(acc, ref)


@pytest.mark.parametrize("d,block", [(1024, 32), (256, 1024 // 4), (512, 64)])
def test_packed_rows_match_table_lookup(cuda, d, block):
    """The row-sharded exchange's device half: rows packed by their owners (in any order),
    then summed / dequantized through positions, equal the plain table lookups bit for bit."""
    rng = np.random.default_rng(d + 3 * block)
    rows, T, H = 3000, 41, 24
    table = rng.integers(0, 256, size=(rows, d), dtype=np.uint8)
    table[(table & 0x7F) == 0x7F] = 0
    scale = rng.integers(112, 130, size=(rows, d // block), dtype=np.uint8)
    idx = _d(rng.integers(0, rows, size=(T, H)))
    emb = q.engram.EngramEmbedding(rows, d, block)
    emb.weight, emb.scale = _d(table), _d(scale)
    ops = q.engram._CudaRowOps()
    perm = torch.from_numpy(rng.permutation(T * H)).cuda()
    ids = idx.reshape(-1)[perm].contiguous()                  # rows in shuffled order
    packed = ops.pack_rows(emb.weight, emb.scale, 0, d, block, ids)
    assert packed.shape == (T * H, ops.row_bytes(d, block))
    pos = torch.empty_like(perm)
    pos[perm] = torch.arange(T * H, device="cuda")            # (t, h) -> packed row
    for dt in (torch.float32, torch.bfloat16):
        out = torch.empty(T, d, dtype=dt, device="cuda")
        ops.sum_rows(packed, pos.reshape(T, H), d, block, out)
        assert torch.equal(out, emb.gather_sum(idx, dt))
        rows_out = torch.empty(T * H, d, dtype=dt, device="cuda")
        ops.dequant_rows(packed, pos, d, block, rows_out)
        assert torch.equal(rows_out, emb(idx, dt).reshape(T * H, d))


def test_packed_rows_off_shard_are_zero(cuda):
    """An owner asked for a row it does not hold packs zeros (codes and scale)."""
    rng = np.random.default_rng(5)
    rows, d, block = 100, 256, 32
    table = _d(rng.integers(1, 126, size=(rows, d), dtype=np.uint8))
    scale = _d(rng.integers(115, 128, size=(rows, d // block), dtype=np.uint8))
    ops = q.engram._CudaRowOps()
    ids = torch.tensor([1000, 1001, 1099, 1100, 999], dtype=torch.int64, device="cuda")
    packed = ops.pack_rows(table, scale, 1000, d, block, ids)
    assert torch.equal(packed[0, :d], table[0]) and torch.equal(packed[2, d:d + d // block], scale[99])
    assert int(packed[3].abs().sum()) == 0 and int(packed[4].abs().sum()) == 0


def test_engram_gate_golden(cuda):
    """The fused gate against upstream Engram.forward (fp32 stream and kv), with and without
    the token mask."""
    g = golden("engram_gate.npz")
    args = types.SimpleNamespace(dim=g["x"].shape[-1], hc_mult=g["x"].shape[-2],
                                 norm_eps=float(g["eps"]), engram_max_ngram_size=4,
                                 engram_n_heads=2, engram_head_dim=16,
                                 engram_num_embeddings=(100,))
    eg = q.engram.Engram(args, 0)
    eg.q_weight, eg.k_weight = _d(g["q_weight"]), _d(g["k_weight"])
    x, kv = _d(g["x"]), _d(g["kv"])
    got = eg.gate(x, kv).cpu().numpy()
    np.testing.assert_allclose(got, g["out"], rtol=1e-5, atol=2e-6)
    got = eg.gate(x, kv, token_mask=_d(g["mask"])).cpu().numpy()
    np.testing.assert_allclose(got, g["out_masked"], rtol=1e-5, atol=2e-6)


def test_engram_module_fp8_wkv(cuda):
    """Rows gathered from an fp8 table -> bf16 -> release-format fp8 wkv -> gate, bf16 stream,
    against the oracle chain (row gather, bf16 rounding, exact decode, float64 projection
    rounded to bf16, the gate)."""
    from gen import bf16_acts, fp8_weight
    from oracle import formats as F
    rng = np.random.default_rng(12)
    rows_n, hd, heads, hc, D, B, Lq = 2000, 256, 2, 4, 256, 3, 7
    cols = 3 * heads
    args = types.SimpleNamespace(dim=D, hc_mult=hc, norm_eps=1e-6, engram_max_ngram_size=4,
                                 engram_n_heads=heads, engram_head_dim=hd,
                                 engram_num_embeddings=(rows_n,))
    table = rng.integers(0, 126, size=(rows_n, hd), dtype=np.uint8)
    scale = rng.integers(115, 124, size=(rows_n, hd // 32), dtype=np.uint8)
    w, s = fp8_weight(rng, (hc + 1) * D, cols * hd, 112, 120)
    qw = (1.0 + 0.1 * rng.standard_normal((hc, D))).astype(np.float32)
    kw = (1.0 + 0.1 * rng.standard_normal((hc, D))).astype(np.float32)
    xb, xf = bf16_acts(rng, B * Lq * hc, D)
    ids = rng.integers(0, rows_n, size=(B, Lq, cols))
    eg = q.engram.Engram(args, 0)
    eg.embed.weight, eg.embed.scale = _d(table), _d(scale)
    eg.wkv = q.linear.FP8Linear(_d(w), _d(s))
    eg.q_weight, eg.k_weight = _d(qw), _d(kw)
    x = _d(xb.view(np.int16)).view(torch.bfloat16).reshape(B, Lq, hc, D)
    got = eg(x, _d(ids)).float().cpu().numpy()
    # oracle chain
    rows = OE.gather_rows(table, scale, ids.reshape(-1), 32).reshape(B * Lq, cols * hd)
    rows = F.bf16_bits_to_f32(F.f32_to_bf16_bits(rows.astype(np.float32)))
    wd = F.dequant_fp8(w, s, "f32").astype(np.float64)
    kv = (rows.astype(np.float64) @ wd.T).astype(np.float32)
    kv = F.bf16_bits_to_f32(F.f32_to_bf16_bits(kv))
    want = OE.engram_gate(xf.reshape(B * Lq, hc, D), kv, qw, kw, 1e-6)
    assert rel_fro(got.reshape(B * Lq, hc, D), want) < 1e-2


# up to 1000 tokens, up to 32 rows a token, a single row, rows off the shard
@pytest.mark.parametrize("d,block,row_lo,T,H", [(1024, 1024, 0, 29, 24), (256, 32, 0, 29, 24),
                                                (512, 64, 700, 29, 24), (1024, 1024, 0, 700, 24),
                                                (1024, 128, 300, 500, 32), (512, 64, 0, 333, 1),
                                                (256, 256, 50, 1000, 7)])
def test_packed_table_lookups_identical(cuda, d, block, row_lo, T, H):
    """A table stored as packed rows (EngramEmbedding.pack) gives the same bits as the codes
    and scales stored apart, for the summed and the per-row lookups; ids outside this shard
    read zero rows either way."""
    rng = np.random.default_rng(d + row_lo + T)
    rows = 3000
    table = rng.integers(0, 256, size=(rows, d), dtype=np.uint8)
    table[(table & 0x7F) == 0x7F] = 0
    scale = rng.integers(112, 130, size=(rows, d // block), dtype=np.uint8)
    idx = _d(rng.integers(row_lo - 50, row_lo + rows + 50, size=(T, H)))
    a = q.engram.EngramEmbedding(rows, d, block, row_lo=row_lo)
    a.weight, a.scale = _d(table), _d(scale)
    b = q.engram.EngramEmbedding(rows, d, block, row_lo=row_lo)
    b.weight, b.scale = _d(table), _d(scale)
    b.pack()
    assert b.weight is None and b.packed.shape[0] == rows
    for dt in (torch.float32, torch.bfloat16):
        if d in (256, 512, 1024):
            assert torch.equal(a.gather_sum(idx, dt), b.gather_sum(idx, dt))
        assert torch.equal(a(idx, dt), b(idx, dt))


@pytest.mark.parametrize("d,block,shard", [(512, 64, False), (1024, 1024, True), (256, 32, False)])
def test_lookup_sum_matches_hash_then_sum(cuda, d, block, shard):
    """The fused hash + row sum (EngramHasher.lookup_sum, one launch) gives the same bits as
    the hasher followed by gather_sum on its ids, for the second of two hash layers, through
    one id cache over two chunks (pad positions at the start, cached ids after), B = 2, fp32
    and bf16 out; the id cache ends the same.  shard: the table holds rows [300, n - 300)
    only, so some ids read zero rows."""
    rng = np.random.default_rng(d + block)
    layer_ids, G, H, vocab = (1, 5), 4, 8, 2000
    primes, offsets = OE.build_layout(len(layer_ids), G, H, vocab)
    sums = primes.reshape(len(layer_ids), -1).sum(-1)
    tm = rng.integers(0, 500, size=1200, dtype=np.int64)
    tm[7] = 499
    args = types.SimpleNamespace(engram_layer_ids=layer_ids,
                                 engram_num_embeddings=tuple(int(v) for v in sums),
                                 engram_max_ngram_size=G, engram_vocab_size=vocab,
                                 engram_n_heads=H, engram_pad_id=2,
                                 engram_compressed_vocab_size=500)
    h = q.engram.EngramHasher(args, tm)
    n = int(sums[1])
    lo, hi = (300, n - 300) if shard else (0, n)
    table = rng.integers(0, 256, size=(hi - lo, d), dtype=np.uint8)
    table[(table & 0x7F) == 0x7F] = 0
    scale = rng.integers(112, 130, size=(hi - lo, d // block), dtype=np.uint8)
    emb = q.engram.EngramEmbedding(hi - lo, d, block, row_lo=lo)
    emb.weight, emb.scale = _d(table), _d(scale)
    emb.pack()
    ids = rng.integers(0, 1200, size=(2, 37), dtype=np.int64)
    L1 = 5
    recips = h._dev["recips"]
    for dt in (torch.float32, torch.bfloat16):
        # given reciprocals, the kernel's own division (NULL reciprocals), the two-launch form
        for given, fused_max in ((True, 4096), (False, 4096), (True, 0)):
            h._dev["recips"] = recips if given else None
            h.fused_max_positions = fused_max
            ca = torch.zeros((2, 64), dtype=torch.int64, device="cuda")
            cb = torch.zeros_like(ca)
            for s0, s1 in ((0, L1), (L1, ids.shape[1])):
                chunk = _d(ids[:, s0:s1])
                got = h.lookup_sum(emb, chunk, s0, ca, layer=1, out_dtype=dt)
                hid = h(chunk, s0, cb)
                want = emb.gather_sum(hid[:, :, 1], dt)
                assert got.shape == (2, s1 - s0, d)
                assert torch.equal(got, want)
                assert torch.equal(ca, cb)
    h._dev["recips"] = recips
    h.fused_max_positions = q.engram.EngramHasher.fused_max_positions
