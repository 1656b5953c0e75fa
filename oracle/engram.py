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
