"""Engram hashing and row lookup restated in numpy.  Test infrastructure only.

Follows deepseek_v41_mlx/engram.py:
  _isprime / find_next_prime   engram.py:35-52
  build_layout                 engram.py:55-75   primes drawn upward from vocab_size-1,
                                                 never reused across (layer, n-gram, head)
  compute_hash_multipliers     engram.py:78-87   default_rng(10007*layer_id), odd, bounded
  EngramHasher.__call__        engram.py:154-180 compressed ids -> id cache (in place),
                                                 lookback with pad at the sequence start,
                                                 int64 products, rolling XOR, % prime + offset
  EngramEmbedding.__call__     engram.py:197-203 row gather + dequant_fp8_rows
and the upstream row-sharded lookup ParallelEngramEmbedding.forward
(docs/reference/model.py:312-325): ids outside the shard read zero rows.
The gather-sum form sums the per-token rows in
hash-column order in fp32.
  Engram.__call__              engram.py:245-264 kv = wkv(rows); per (token, hc copy)
                                                 normalised dot of the stream with the key,
                                                 signed-sqrt sigmoid gate, h + gate * value
(upstream Engram.forward, docs/reference/model.py:344-365, adds the token mask).
"""

from __future__ import annotations

import numpy as np

from .formats import dequant_fp8_rows, to_dtype


def isprime(n: int) -> bool:
    if n < 2:
        return False
    if n % 2 == 0:
        return n == 2
    i = 3
    while i * i <= n:
        if n % i == 0:
            return False
        i += 2
    return True


def find_next_prime(start: int, seen: set) -> int:
    c = start + 1
    while not isprime(c) or c in seen:
        c += 1
    return c


def build_layout(n_layers: int, max_ngram: int, n_heads: int, vocab_size: int):
    """-> primes int64 [nL, G-1, H], offsets int64 [nL, (G-1)*H]."""
    primes, seen = [], set()
    for _ in range(n_layers):
        per_ngram = []
        for _ in range(max_ngram - 1):
            sizes, cur = [], vocab_size - 1
            for _ in range(n_heads):
                cur = find_next_prime(cur, seen)
                seen.add(cur)
                sizes.append(cur)
            per_ngram.append(sizes)
        primes.append(per_ngram)
    flat = [[p for g in layer for p in g] for layer in primes]
    offsets = [np.cumsum([0, *f[:-1]]) for f in flat]
    return np.asarray(primes, dtype=np.int64), np.asarray(offsets, dtype=np.int64)


def compute_hash_multipliers(layer_ids, max_ngram: int, compressed_vocab: int) -> np.ndarray:
    max_long = np.iinfo(np.int64).max
    bound = max(1, (max_long // compressed_vocab) // 2)
    rows = []
    for lid in layer_ids:
        g = np.random.default_rng(10007 * lid)
        v = g.integers(low=0, high=bound, size=(max_ngram,), dtype=np.int64)
        rows.append(v * 2 + 1)
    return np.stack(rows)


def engram_hash(input_ids, start_pos, ids_cache, token_map, multipliers, primes, offsets,
                pad_id: int, max_ngram: int):
    """engram.py:154-180.  Writes ids_cache[:B, start:start+L] in place; returns
    int64 [B, L, nL, (G-1)*H]."""
    input_ids = np.asarray(input_ids)
    B, L = input_ids.shape
    comp = np.asarray(token_map, dtype=np.int64)[input_ids]
    ids_cache[:B, start_pos:start_pos + L] = comp
    pos = np.broadcast_to(np.arange(start_pos, start_pos + L), (B, L))
    toks, blocked = [], np.zeros((B, L), dtype=bool)
    for shift in range(max_ngram):
        src = np.take_along_axis(ids_cache[:B], np.clip(pos - shift, 0, None), axis=1)
        blocked = blocked | (pos < shift)
        toks.append(np.where(blocked, pad_id, src))
    toks = np.stack(toks, -1)                                   # [B, L, G]
    prod = toks[:, :, None, :] * multipliers                    # [B, L, nL, G]
    rolling, hashes = prod[..., 0], []
    for i in range(1, max_ngram):
        rolling = np.bitwise_xor(rolling, prod[..., i])
        hashes.append(rolling[..., None] % primes[:, i - 1])
    return np.concatenate(hashes, -1) + offsets


def gather_rows(table, scale, idx, block, row_lo=0):
    """EngramEmbedding.__call__ (engram.py:197-203) on a row shard starting at
    row_lo; ids outside the shard give zero rows (model.py:312-325)."""
    idx = np.asarray(idx, dtype=np.int64)
    rows = table.shape[0]
    local = idx - row_lo
    mask = (local < 0) | (local >= rows)
    local = np.where(mask, 0, local)
    v = dequant_fp8_rows(table[local], scale[local], block)
    v[mask] = 0.0
    return v


def gather_sum(table, scale, idx, block, out_dtype="bf16", row_lo=0):
    """idx [T, n] -> out [T, d]: fp32 sum over the n rows in column order."""
    rows = gather_rows(table, scale, idx, block, row_lo)       # [T, n, d]
    acc = np.zeros((rows.shape[0], rows.shape[2]), dtype=np.float32)
    for h in range(rows.shape[1]):
        acc = (acc + rows[:, h]).astype(np.float32)
    return to_dtype(acc, out_dtype)


def engram_gate(x, kv, q_weight, k_weight, eps, clamp=1e-6, token_mask=None):
    """Engram.__call__ after the wkv projection (engram.py:248-264), fp32.

    x [..., hc, dim]; kv [..., (hc + 1) * dim] (hc keys, then the shared value);
    q_weight, k_weight [hc, dim].  rstd = rsqrt(mean(h^2) + eps) * rsqrt(mean(key^2) + eps)
    per (token, hc copy); dot = sum(h * (q*k) * key) * rstd / sqrt(dim);
    gate = sigmoid(sign(dot) * sqrt(max(|dot|, clamp))); out = h + gate * value.
    token_mask [...] (upstream model.py:361-362): False closes the gate."""
    x = np.asarray(x, dtype=np.float32)
    kv = np.asarray(kv, dtype=np.float32)
    hc, dim = x.shape[-2], x.shape[-1]
    key = kv[..., :hc * dim].reshape(kv.shape[:-1] + (hc, dim))
    value = kv[..., hc * dim:]
    weight = (np.asarray(q_weight, np.float32) * np.asarray(k_weight, np.float32)).astype(np.float32)
    ms_h = np.mean(np.square(x), axis=-1, dtype=np.float32)
    ms_k = np.mean(np.square(key), axis=-1, dtype=np.float32)
    rstd = (1.0 / np.sqrt(ms_h + np.float32(eps))) * (1.0 / np.sqrt(ms_k + np.float32(eps)))
    dot = np.sum(x * weight * key, axis=-1, dtype=np.float32) * rstd.astype(np.float32) \
        * np.float32(dim ** -0.5)
    mag = np.sqrt(np.maximum(np.abs(dot), np.float32(clamp)))
    gate = 1.0 / (1.0 + np.exp(-np.where(dot < 0, -mag, mag)))
    if token_mask is not None:
        gate = np.where(np.asarray(token_mask)[..., None], gate, 0.0)
    return (x + gate.astype(np.float32)[..., None] * value[..., None, :]).astype(np.float32)
