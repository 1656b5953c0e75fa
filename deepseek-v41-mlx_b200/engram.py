"""Engram hashing and fp8 row lookup on the GPU -- drop-in for deepseek_v41_mlx/engram.py.

* ``build_layout`` / ``compute_hash_multipliers`` / ``find_next_prime`` are the
  reference's host-side setup (engram.py:35-87), restated here in numpy (they
  run once per model, not per token).
* ``EngramHasher(args, token_map)(input_ids, start_pos, ids_cache)`` runs on the
  GPU (engram.py:154-180).  ``ids_cache`` is updated in place as the reference
  does; a numpy cache is accepted and written back.
* ``EngramEmbedding(num, dim, block)(indices)`` gathers e4m3 rows and their ue8m0
  scales and returns fp32 rows (engram.py:197-203).  ``row_lo`` makes it the
  row-sharded ParallelEngramEmbedding (docs/reference/model.py:296-325): ids
  outside [row_lo, row_lo + rows) give zero rows.
* ``QuantizedEngramEmbedding`` is the MLX affine table (engram.py:206-223).
* ``Engram(args, layer_hash_index)(x, hash_ids)`` is the gated write of the looked-up
  rows into the hc-expanded stream (engram.py:225-264): rows -> ``wkv`` (any linear of
  this package, e.g. ``linear.FP8Linear`` for the release's fp8 blocks) -> the fused gate
  kernel ``dsv41_engram_gate``.
* ``gather_sum`` is the summed form used by the benchmark configuration.
* ``ParallelEngramEmbedding(num, dim, block)`` is upstream's row-sharded table
  (docs/reference/model.py:296-325) over a torch.distributed process group: each
  rank keeps ceil(num / world) rows, the raw rows a token needs travel from their
  owners to the rank that handles the token (one all-to-all), and the results are
  all-gathered -- bit-identical to one GPU, unlike a sum of partial sums.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L


def _isprime(n: int) -> bool:
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
    while not _isprime(c) or c in seen:
        c += 1
    return c


def build_layout(args):
    """engram.py:55-75 -> (primes int64 [nL, G-1, H], offsets int64 [nL, (G-1)*H])."""
    primes, seen = [], set()
    for _ in args.engram_layer_ids:
        per = []
        for _ in range(args.engram_max_ngram_size - 1):
            sizes, cur = [], args.engram_vocab_size - 1
            for _ in range(args.engram_n_heads):
                cur = find_next_prime(cur, seen)
                seen.add(cur)
                sizes.append(cur)
            per.append(sizes)
        primes.append(per)
    flat = [[p for g in layer for p in g] for layer in primes]
    offsets = [np.cumsum([0, *f[:-1]]) for f in flat]
    return np.asarray(primes, dtype=np.int64), np.asarray(offsets, dtype=np.int64)


def compute_hash_multipliers(layer_ids, max_ngram_size: int, compressed_vocab_size: int):
    """engram.py:78-87 -- one odd multiplier per (layer, lookback)."""
    max_long = np.iinfo(np.int64).max
    bound = max(1, (max_long // compressed_vocab_size) // 2)
    rows = []
    for lid in layer_ids:
        g = np.random.default_rng(10007 * lid)
        rows.append(g.integers(low=0, high=bound, size=(max_ngram_size,), dtype=np.int64) * 2 + 1)
    return np.stack(rows)


class EngramHasher:
    """engram.py:127-180 on the GPU."""

    def __init__(self, args, token_map, device=None):
        t = L.torch()
        self.args = args
        self.max_ngram = args.engram_max_ngram_size
        tm = np.asarray(token_map, dtype=np.int64)
        n_compressed = int(tm.max()) + 1
        if args.engram_compressed_vocab_size and n_compressed != args.engram_compressed_vocab_size:
            raise ValueError(
                f"compressed vocab {n_compressed} != config {args.engram_compressed_vocab_size}; "
                f"every hash multiplier is derived from it, so a mismatch silently rehashes the table")
        self.pad_id = int(tm[args.engram_pad_id])
        self.primes, self.offsets = build_layout(args)
        self.multipliers = compute_hash_multipliers(args.engram_layer_ids, self.max_ngram,
                                                    n_compressed)
        sums = self.primes.reshape(len(args.engram_layer_ids), -1).sum(-1)
        if tuple(int(s) for s in sums) != tuple(args.engram_num_embeddings):
            raise ValueError(f"prime sums {sums} != engram_num_embeddings "
                             f"{args.engram_num_embeddings}")
        dev = device or t.device("cuda", t.cuda.current_device())
        # floor((2^64 - 1) / p) per prime (the Barrett multipliers), as int64 bit patterns
        recips = np.array([(2 ** 64 - 1) // int(p) if p > 1 else 0 for p in self.primes.flat],
                          dtype=np.uint64).view(np.int64)
        self._dev = {k: t.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in (
            ("token_map", tm), ("mult", self.multipliers), ("primes", self.primes),
            ("offsets", self.offsets), ("recips", recips))}
        self.vocab = len(tm)

    def __call__(self, input_ids, start_pos: int, ids_cache):
        t = L.torch()
        dev = self._dev["token_map"].device
        host_cache = isinstance(ids_cache, np.ndarray)
        cache = t.from_numpy(ids_cache).to(dev) if host_cache else L.cuda_tensor(ids_cache)
        if cache.dtype != t.int64:
            raise ValueError("ids_cache must be int64")
        ids = input_ids if isinstance(input_ids, t.Tensor) else t.as_tensor(np.asarray(input_ids))
        ids = ids.to(dev, dtype=t.int64).contiguous()
        B, Lq = ids.shape
        nL = len(self.args.engram_layer_ids)
        G, H = self.max_ngram, self.args.engram_n_heads
        out = t.empty((B, Lq, nL, (G - 1) * H), dtype=t.int64, device=dev)
        L.call("dsv41_engram_hash", L.ptr(ids), B, Lq, int(start_pos), L.ptr(self._dev["token_map"]),
               self.vocab, L.ptr(cache), cache.shape[1], L.ptr(self._dev["mult"]),
               L.ptr(self._dev["primes"]), L.ptr(self._dev["offsets"]), nL, G, H, self.pad_id,
               L.ptr(out), L.stream_of(out))
        if host_cache:
            ids_cache[...] = cache.cpu().numpy()
        elif cache.data_ptr() != L.as_tensor(ids_cache).data_ptr():
            ids_cache.copy_(cache)
        return out

    # Up to this many positions a call, lookup_sum hashes and sums in one launch; above it the
    # hasher and the gather-sum run apart (measured on B200 with a 1 KB-row table: one launch
    # 12 vs 20 us at 1 to 64 positions, 44 vs 47 us at 4096, 78 vs 76 us at 8192).
    fused_max_positions = 4096

    def lookup_sum(self, embedding, input_ids, start_pos: int, ids_cache, layer: int = 0,
                   out_dtype=None):
        """``embedding.gather_sum(self(input_ids, start_pos, ids_cache)[:, :, layer])``, the
        same bits and the same id-cache update, in one launch where it pays: the hashes are
        computed where the rows are summed and never written.
          * ``EngramEmbedding`` with packed rows (``pack``): ``dsv41_engram_lookup_sum`` up to
            ``fused_max_positions`` positions;
          * ``ParallelEngramEmbedding`` reading its peers' shards in place:
            ``dsv41_engram_lookup_sum_peers`` up to its ``replicate_max_tokens`` positions
            (every rank sums every position; no collective);
        otherwise the hasher and ``gather_sum`` run apart.  -> [B, L, dim]."""
        t = L.torch()
        odt = out_dtype or t.bfloat16
        n_pos = int(np.prod(getattr(input_ids, "shape", np.shape(input_ids))))
        packed = getattr(embedding, "packed", None) is not None
        peers = (isinstance(embedding, ParallelEngramEmbedding) and embedding.peers
                 and embedding.dim in (256, 512, 1024))
        if packed:
            fused = n_pos <= self.fused_max_positions
        elif peers:
            fused = n_pos <= embedding.replicate_max_tokens
        elif isinstance(embedding, EngramEmbedding):
            raise ValueError("lookup_sum reads packed rows: call embedding.pack() first")
        else:
            fused = False
        dev = self._dev["token_map"].device
        if not fused:
            hid = self(input_ids, start_pos, ids_cache)
            return embedding.gather_sum(hid[:, :, layer], odt)
        host_cache = isinstance(ids_cache, np.ndarray)
        cache = t.from_numpy(ids_cache).to(dev) if host_cache else L.cuda_tensor(ids_cache)
        if cache.dtype != t.int64:
            raise ValueError("ids_cache must be int64")
        ids = input_ids if isinstance(input_ids, t.Tensor) else t.as_tensor(np.asarray(input_ids))
        ids = ids.to(dev, dtype=t.int64).contiguous()
        B, Lq = ids.shape
        nL = len(self.args.engram_layer_ids)
        G, H = self.max_ngram, self.args.engram_n_heads
        out = t.empty((B, Lq, embedding.dim), dtype=odt, device=dev)
        hash_args = (L.ptr(ids), B, Lq, int(start_pos), L.ptr(self._dev["token_map"]), self.vocab,
                     L.ptr(cache), cache.shape[1], L.ptr(self._dev["mult"]),
                     L.ptr(self._dev["primes"]), L.ptr(self._dev["offsets"]),
                     L.ptr(self._dev["recips"]), nL, int(layer), G, H, self.pad_id)
        if packed:
            pk = embedding.packed
            L.call("dsv41_engram_lookup_sum", *hash_args, L.ptr(pk), pk.shape[0],
                   embedding.row_lo, embedding.dim, embedding.block, L.dtype_code(odt),
                   L.ptr(out), L.stream_of(out))
        else:
            tabs, scs = embedding._map_peers(dev)[:2]
            L.call("dsv41_engram_lookup_sum_peers", *hash_args, L.ptr(tabs), L.ptr(scs),
                   embedding.world, embedding.part, embedding.num_embeddings, embedding.dim,
                   embedding.block, L.dtype_code(odt), L.ptr(out), L.stream_of(out))
        if host_cache:
            ids_cache[...] = cache.cpu().numpy()
        elif cache.data_ptr() != L.as_tensor(ids_cache).data_ptr():
            ids_cache.copy_(cache)
        return out


class EngramEmbedding:
    """engram.py:183-203: e4m3 table [rows, d] + ue8m0 [rows, d/block] -> fp32 rows."""

    def __init__(self, num_embeddings: int, dim: int, block: int = 32, row_lo: int = 0):
        self.num_embeddings, self.dim, self.block, self.row_lo = num_embeddings, dim, block, row_lo
        self.weight = None
        self.scale = None
        self.packed = None       # [rows, row_bytes]: codes then scales, one read a row

    def pack(self, keep=False):
        """Store the table as packed rows (codes then the row's scale bytes, padded to 16:
        1040 bytes a row at dim 1024, +1.6%), so that every lookup reads one contiguous row
        instead of the row and, elsewhere, its scale (measured 22-30% faster on random rows).
        ``keep=False`` drops the references to ``weight`` / ``scale``."""
        t = L.torch()
        w = L.u8(L.cuda_tensor(self.weight, "weight"))
        s = L.u8(L.cuda_tensor(self.scale, "scale"))
        rb = int(L.load().dsv41_engram_row_bytes(self.dim, self.block))
        self.packed = t.empty((w.shape[0], rb), dtype=t.uint8, device=w.device)
        L.call("dsv41_engram_pack_rows", L.ptr(w), L.ptr(s), w.shape[0], 0, self.dim, self.block,
               None, w.shape[0], L.ptr(self.packed), L.stream_of(w))
        if not keep:
            self.weight = self.scale = None
        return self

    def _packed_ids(self, idx):
        return idx if self.row_lo == 0 else idx - self.row_lo

    def __call__(self, indices, out_dtype=None):
        t = L.torch()
        if self.packed is not None:
            idx = L.cuda_tensor(indices, "indices").to(t.int64).contiguous()
            odt = out_dtype or t.float32
            out = t.empty(tuple(idx.shape) + (self.dim,), dtype=odt, device=idx.device)
            pos = self._packed_ids(idx).contiguous()
            L.call("dsv41_engram_dequant_rows", L.ptr(self.packed), self.packed.shape[0],
                   self.dim, self.block, L.ptr(pos), pos.numel(), L.dtype_code(odt), L.ptr(out),
                   L.stream_of(idx))
            return out
        w = L.u8(L.cuda_tensor(self.weight, "weight"))
        s = L.u8(L.cuda_tensor(self.scale, "scale"))
        idx = L.cuda_tensor(indices, "indices").to(t.int64)
        odt = out_dtype or t.float32
        out = t.empty(tuple(idx.shape) + (self.dim,), dtype=odt, device=idx.device)
        L.call("dsv41_engram_gather_rows", L.ptr(w), L.ptr(s), w.shape[0], self.row_lo, self.dim,
               self.block, L.ptr(idx), idx.numel(), L.dtype_code(odt), L.ptr(out),
               L.stream_of(idx))
        return out

    def gather_sum(self, indices, out_dtype=None):
        """indices [..., n] -> [..., d]: fp32 sum of each token's n rows in column order."""
        t = L.torch()
        if self.packed is not None:
            idx = L.cuda_tensor(indices, "indices").to(t.int64)
            n = idx.shape[-1]
            n_tok = idx.numel() // n
            odt = out_dtype or t.bfloat16
            out = t.empty(tuple(idx.shape[:-1]) + (self.dim,), dtype=odt, device=idx.device)
            pos = self._packed_ids(idx).contiguous()
            L.call("dsv41_engram_sum_rows", L.ptr(self.packed), self.packed.shape[0], self.dim,
                   self.block, L.ptr(pos), n_tok, n, L.dtype_code(odt), L.ptr(out),
                   L.stream_of(idx))
            return out
        w = L.u8(L.cuda_tensor(self.weight, "weight"))
        s = L.u8(L.cuda_tensor(self.scale, "scale"))
        idx = L.cuda_tensor(indices, "indices").to(t.int64)
        n = idx.shape[-1]
        n_tok = idx.numel() // n
        odt = out_dtype or t.bfloat16
        out = t.empty(tuple(idx.shape[:-1]) + (self.dim,), dtype=odt, device=idx.device)
        L.call("dsv41_engram_gather_sum", L.ptr(w), L.ptr(s), w.shape[0], self.row_lo, self.dim,
               self.block, L.ptr(idx), n_tok, n, L.dtype_code(odt), L.ptr(out), L.stream_of(idx))
        return out


class QuantizedEngramEmbedding:
    """engram.py:206-223: MLX affine table, rows dequantized on lookup (fp32 out)."""

    def __init__(self, num_embeddings: int, dim: int, group_size: int = 64, bits: int = 4):
        self.group_size, self.bits, self.dim = group_size, bits, dim
        self.weight = self.scales = self.biases = None

    def __call__(self, indices):
        from .dequant import dequantize_affine
        t = L.torch()
        idx = L.cuda_tensor(indices, "indices").to(t.int64).reshape(-1)
        w = L.cuda_tensor(self.weight).index_select(0, idx)
        s = L.cuda_tensor(self.scales).index_select(0, idx)
        b = L.cuda_tensor(self.biases).index_select(0, idx)
        out = dequantize_affine(w, s, b, self.group_size, self.bits, t.float32)
        return out.reshape(tuple(indices.shape) + (self.dim,))


class _CudaRowOps:
    """The device half of ParallelEngramEmbedding: libdsv41q's row pack / sum / dequant."""

    def row_bytes(self, d, block):
        return int(L.load().dsv41_engram_row_bytes(d, block))

    def pack_rows(self, weight, scale, row_lo, d, block, ids):
        t = L.torch()
        rb = self.row_bytes(d, block)
        out = t.empty((ids.numel(), rb), dtype=t.uint8, device=ids.device)
        L.call("dsv41_engram_pack_rows", L.ptr(weight), L.ptr(scale), weight.shape[0], row_lo, d,
               block, L.ptr(ids), ids.numel(), L.ptr(out), L.stream_of(ids))
        return out

    def sum_rows(self, recv, pos, d, block, out):
        n_tok, n = pos.shape
        L.call("dsv41_engram_sum_rows", L.ptr(recv) if recv.numel() else None, recv.shape[0], d,
               block, L.ptr(pos), n_tok, n, L.dtype_code(out.dtype), L.ptr(out), L.stream_of(out))

    def dequant_rows(self, recv, pos, d, block, out):
        L.call("dsv41_engram_dequant_rows", L.ptr(recv) if recv.numel() else None, recv.shape[0],
               d, block, L.ptr(pos), pos.numel(), L.dtype_code(out.dtype), L.ptr(out),
               L.stream_of(out))


class ParallelEngramEmbedding:
    """Upstream ParallelEngramEmbedding (docs/reference/model.py:296-325) over a process group.

    Rank r holds rows [r * part, (r + 1) * part) of the table, part = ceil(num / world)
    (``weight`` u8 e4m3 [part, dim], ``scale`` u8 ue8m0 [part, dim / block]).  The indices
    are the same on every rank (the hasher runs everywhere), so every rank can tell, with
    no request message, which of its rows each token needs.  Rank r handles tokens
    [r * per, (r + 1) * per): the owners pack the raw rows those tokens need, one
    all_to_all_single delivers them, rank r dequantizes (``__call__``) or sums them per
    token in head order (``gather_sum``), and all_gather_into_tensor gives every rank the
    whole result.  Upstream's masked lookup + all_reduce gives the same rows; this moves
    the fp8 rows once instead of reducing bf16 rows over all ranks.  On CUDA the shards are
    read in place over NVLink instead (peer mappings); there, up to
    ``replicate_max_tokens`` tokens every rank sums all of them and no collective runs.
    """

    def __init__(self, num_embeddings: int, dim: int, block: int = 32, rank=None, world=None,
                 group=None, ops=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        init = dist.is_available() and dist.is_initialized()
        self.world = world if world is not None else (dist.get_world_size(group) if init else 1)
        self.rank = rank if rank is not None else (dist.get_rank(group) if init else 0)
        self.num_embeddings, self.dim, self.block = num_embeddings, dim, block
        self.part = -(-num_embeddings // self.world)
        self.row_lo = self.rank * self.part
        self.weight = None
        self.scale = None
        self.ops = ops if ops is not None else _CudaRowOps()
        self.peers = ops is None          # CUDA shards: read peers' rows in place (NVLink)
        self._peer = None                 # (table ptrs, scale ptrs, mapped bases, key)

    def plan(self, idx2):
        """idx2 int64 [T, H] (same on every rank) -> the exchange for this rank.

        send_ids: global row ids this rank owns, in (token, head) order, grouped by the
        handling rank; recv_pos[(t - t0) * H + h]: row of (t, h) in the receive buffer
        (grouped by owner rank, (token, head) order inside a group)."""
        t = L.torch()
        T, H = idx2.shape
        ws, r = self.world, self.rank
        dev = idx2.device
        per = max(1, -(-T // ws))
        owner = t.div(idx2.reshape(-1), self.part, rounding_mode="floor").clamp_(0, ws - 1)
        tok = t.arange(T, device=dev).repeat_interleave(H)
        mine = (owner == r).nonzero(as_tuple=True)[0]
        send_ids = idx2.reshape(-1)[mine].contiguous()
        send_counts = t.bincount(t.div(tok[mine], per, rounding_mode="floor"), minlength=ws)
        t0 = min(T, r * per)
        t1 = min(T, t0 + per)
        my = owner[t0 * H:t1 * H]
        order = t.sort(my, stable=True).indices
        recv_pos = t.empty_like(order)
        recv_pos[order] = t.arange(order.numel(), device=dev)
        recv_counts = t.bincount(my, minlength=ws)
        counts = t.cat([send_counts, recv_counts]).tolist()          # one host sync
        return {"T": T, "H": H, "per": per, "t0": t0, "t1": t1, "send_ids": send_ids,
                "send_counts": counts[:ws], "recv_counts": counts[ws:],
                "recv_pos": recv_pos.reshape(t1 - t0, H)}

    def _exchange(self, idx2):
        t = L.torch()
        plan = self.plan(idx2)
        rb = self.ops.row_bytes(self.dim, self.block)
        send = self.ops.pack_rows(self.weight, self.scale, self.row_lo, self.dim, self.block,
                                  plan["send_ids"])
        recv = t.empty((sum(plan["recv_counts"]), rb), dtype=t.uint8, device=idx2.device)
        self.dist.all_to_all_single(recv.reshape(-1), send.reshape(-1),
                                    [c * rb for c in plan["recv_counts"]],
                                    [c * rb for c in plan["send_counts"]], group=self.group)
        return plan, recv

    def _gather_all(self, part_out, n_total):
        t = L.torch()
        full = t.empty((part_out.shape[0] * self.world,) + tuple(part_out.shape[1:]),
                       dtype=part_out.dtype, device=part_out.device)
        self.dist.all_gather_into_tensor(full, part_out, group=self.group)
        return full[:n_total]

    # ------------------------------------------------------------ peer-memory form
    def _map_peers(self, dev):
        """Map every rank's shard (codes and scales) into this process (collective, once; call
        remap() after replacing ``weight`` / ``scale``)."""
        t = L.torch()
        lib = L.load()
        w = L.u8(L.cuda_tensor(self.weight, "weight"))
        sc = L.u8(L.cuda_tensor(self.scale, "scale"))
        key = (w.data_ptr(), sc.data_ptr())
        if self._peer is not None and self._peer[3] == key:
            return self._peer
        need = max(0, min(self.part, self.num_embeddings - self.rank * self.part))
        if w.shape[0] < need or sc.shape[0] < need:
            raise ValueError(f"shard has {w.shape[0]} rows, expected {need} (of {self.part})")
        nb = int(lib.dsv41_ep_handle_bytes())
        rec = []
        for a in (w, sc):
            h = (C.c_uint8 * nb)()
            off = C.c_int64(0)
            L.call("dsv41_ipc_export", L.ptr(a), C.cast(h, C.c_void_p), C.byref(off))
            rec.append(bytes(h) + int(off.value).to_bytes(8, "little"))
        mine = t.tensor(list(rec[0] + rec[1]), dtype=t.uint8, device=dev)
        every = t.empty(mine.numel() * self.world, dtype=t.uint8, device=dev)
        self.dist.all_gather_into_tensor(every, mine, group=self.group)
        allb = bytes(every.cpu().numpy().tobytes())
        per = len(rec[0])
        opened = {}                       # handle bytes -> mapped base (one import each)
        ptrs = [[], []]
        for r in range(self.world):
            for j, a in enumerate((w, sc)):
                blob = allb[(2 * r + j) * per:(2 * r + j + 1) * per]
                if r == self.rank:
                    ptrs[j].append(a.data_ptr())
                    continue
                hnd, off = blob[:nb], int.from_bytes(blob[nb:], "little")
                if hnd not in opened:
                    base = C.c_void_p()
                    hb = (C.c_uint8 * nb).from_buffer_copy(hnd)
                    L.call("dsv41_ipc_import", C.cast(hb, C.c_void_p), C.byref(base))
                    opened[hnd] = base.value
                ptrs[j].append(opened[hnd] + off)
        tabs = t.tensor(ptrs[0], dtype=t.int64, device=dev)
        scs = t.tensor(ptrs[1], dtype=t.int64, device=dev)
        self.dist.barrier(group=self.group)
        self._peer = (tabs, scs, list(opened.values()), key, w, sc)
        return self._peer

    def remap(self):
        """Unmap the peers' shards (collective); the next lookup maps them again."""
        if self._peer is not None:
            L.torch().cuda.synchronize()
            self.dist.barrier(group=self.group)
            for base in self._peer[2]:
                L.call("dsv41_ipc_close", base)
            self._peer = None

    # Up to this many tokens a call, every rank sums all of them from the shards in place and
    # no collective runs (a T=1 lookup is then a few NVLink row reads); above it each rank
    # sums its slice of the tokens and the slices are all-gathered, so that no rank reads
    # every row.  Same kernel, same rows, same order either way.
    replicate_max_tokens = 64

    def _peer_sum(self, idx2, odt):
        """The tokens summed from the shards in place: all of them on every rank (small T),
        or this rank's slice, then all-gathered."""
        t = L.torch()
        tabs, scs = self._map_peers(idx2.device)[:2]
        T, H = idx2.shape
        if T <= self.replicate_max_tokens:
            out = t.empty((T, self.dim), dtype=odt, device=idx2.device)
            sl = idx2.contiguous()
            L.call("dsv41_engram_gather_sum_peers", L.ptr(tabs), L.ptr(scs), self.world,
                   self.part, self.num_embeddings, self.dim, self.block, L.ptr(sl), T, H,
                   L.dtype_code(odt), L.ptr(out), L.stream_of(sl))
            return out
        per = max(1, -(-T // self.world))
        t0 = min(T, self.rank * per)
        t1 = min(T, t0 + per)
        part_out = t.zeros((per, self.dim), dtype=odt, device=idx2.device)
        if t1 > t0:
            sl = idx2[t0:t1].contiguous()
            L.call("dsv41_engram_gather_sum_peers", L.ptr(tabs), L.ptr(scs), self.world,
                   self.part, self.num_embeddings, self.dim, self.block, L.ptr(sl), t1 - t0, H,
                   L.dtype_code(odt),
                   L.ptr(part_out), L.stream_of(sl))
        return self._gather_all(part_out, T)

    def gather_sum(self, indices, out_dtype=None):
        """indices [..., H] -> [..., dim]: each token's H rows summed in head order (fp32)."""
        t = L.torch()
        idx2 = indices.reshape(-1, indices.shape[-1]).to(t.int64)
        if self.peers and idx2.is_cuda and self.dim in (256, 512, 1024):
            out = self._peer_sum(idx2, out_dtype or t.bfloat16)
            return out.reshape(tuple(indices.shape[:-1]) + (self.dim,))
        plan, recv = self._exchange(idx2)
        odt = out_dtype or t.bfloat16
        part_out = t.zeros((plan["per"], self.dim), dtype=odt, device=idx2.device)
        n_my = plan["t1"] - plan["t0"]
        if n_my:
            self.ops.sum_rows(recv, plan["recv_pos"], self.dim, self.block, part_out[:n_my])
        out = self._gather_all(part_out, plan["T"])
        return out.reshape(tuple(indices.shape[:-1]) + (self.dim,))

    def __call__(self, indices, out_dtype=None):
        """indices [...] -> [..., dim] rows (bf16 as upstream returns them)."""
        t = L.torch()
        idx2 = indices.reshape(-1, 1).to(t.int64)
        if self.peers and idx2.is_cuda and self.dim in (256, 512, 1024):
            out = self._peer_sum(idx2, out_dtype or t.bfloat16)     # one row per "token"
            return out.reshape(tuple(indices.shape) + (self.dim,))
        plan, recv = self._exchange(idx2)
        odt = out_dtype or t.bfloat16
        part_out = t.zeros((plan["per"], self.dim), dtype=odt, device=idx2.device)
        n_my = plan["t1"] - plan["t0"]
        if n_my:
            self.ops.dequant_rows(recv, plan["recv_pos"].reshape(-1), self.dim, self.block,
                                  part_out[:n_my])
        out = self._gather_all(part_out, plan["T"])
        return out.reshape(tuple(indices.shape) + (self.dim,))


class Engram:
    """engram.py:225-264 (upstream Engram, docs/reference/model.py:328-365): the n-gram rows,
    projected by ``wkv`` to one key per hc copy plus a shared value, written into the
    hc-expanded stream x [..., hc, dim] through a gate -- the normalised dot of the stream
    with the key, signed square root, sigmoid.  ``wkv`` is a linear of this package
    (``linear.FP8Linear`` for the release's fp8 32x32 blocks, ``linear.QuantizedLinear`` for
    MLX affine); ``q_weight`` / ``k_weight`` [hc, dim] default to ones as in the reference."""

    def __init__(self, args, layer_hash_index: int):
        self.layer_hash_index = layer_hash_index
        self.dim = args.dim
        self.hc_mult = args.hc_mult
        self.eps = float(args.norm_eps)
        self.clamp_value = 1e-6
        self.n_hash_cols = (args.engram_max_ngram_size - 1) * args.engram_n_heads
        self.head_dim = args.engram_head_dim
        self.embed = EngramEmbedding(args.engram_num_embeddings[layer_hash_index],
                                     args.engram_head_dim, getattr(args, "engram_block", 32))
        self.wkv = None
        self.q_weight = None
        self.k_weight = None

    def _qk(self, device):
        t = L.torch()
        ones = t.ones((self.hc_mult, self.dim), dtype=t.float32, device=device)
        q = ones if self.q_weight is None else L.cuda_tensor(self.q_weight).float().contiguous()
        k = ones if self.k_weight is None else L.cuda_tensor(self.k_weight).float().contiguous()
        return q, k

    def gate(self, x, kv, token_mask=None):
        """The gated write for a given kv [..., (hc + 1) * dim] (the step after wkv)."""
        t = L.torch()
        xt = L.cuda_tensor(x, "x")
        if xt.dtype not in (t.float32, t.bfloat16):
            xt = xt.to(t.bfloat16)
        xt = xt.contiguous()
        kvt = L.cuda_tensor(kv, "kv")
        if kvt.dtype not in (t.float32, t.bfloat16):
            kvt = kvt.float()
        kvt = kvt.contiguous()
        hc, D = self.hc_mult, self.dim
        if tuple(xt.shape[-2:]) != (hc, D) or kvt.shape[-1] != (hc + 1) * D:
            raise ValueError(f"x [..., {hc}, {D}] and kv [..., {(hc + 1) * D}] expected")
        T = xt.numel() // (hc * D)
        q, k = self._qk(xt.device)
        m = None
        if token_mask is not None:
            m = L.cuda_tensor(token_mask, "token_mask").to(t.uint8).reshape(-1).contiguous()
        out = t.empty_like(xt)
        L.call("dsv41_engram_gate", L.ptr(xt), L.dtype_code(xt.dtype), L.ptr(kvt),
               L.dtype_code(kvt.dtype), L.ptr(q), L.ptr(k), L.ptr(m) if m is not None else None,
               T, hc, D, self.eps, self.clamp_value, L.ptr(out), L.stream_of(xt))
        return out

    def __call__(self, x, hash_ids, token_mask=None):
        """x [B, L, hc, dim]; hash_ids [B, L, n_hash_cols] -> the updated stream, x's dtype."""
        t = L.torch()
        if self.wkv is None:
            raise ValueError("Engram.wkv is not set")
        xt = L.cuda_tensor(x, "x")
        dt = xt.dtype if xt.dtype in (t.float32, t.bfloat16) else t.bfloat16
        ids = L.cuda_tensor(hash_ids, "hash_ids").to(t.int64)
        rows = self.embed(ids, dt)                                    # rows cast to x's dtype
        rows = rows.reshape(-1, self.n_hash_cols * self.head_dim)
        kv = self.wkv(rows, out_dtype=dt)                             # the linear's output dtype
        return self.gate(xt, kv.reshape(tuple(xt.shape[:-2]) + (-1,)), token_mask)
