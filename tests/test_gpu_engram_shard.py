"""Row-sharded engram table on 2 GPUs (NCCL) vs the whole table on one GPU: bit-exact.

Each rank holds half the rows (ceil split); the hashed indices are the same on both ranks.
The summed lookup (gather_sum) and the per-row lookup (upstream ParallelEngramEmbedding's
output) must equal the single-table results on every rank.  Skipped with fewer than 2 GPUs.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _lookup_sum_check(engram, dev):
    """EngramHasher.lookup_sum on the sharded table (one launch reading the peers' shards
    up to replicate_max_tokens positions, hasher + gather_sum above) == hasher + gather_sum
    on the whole table, bits and id cache, over three chunks through one cache."""
    import types
    import numpy as np
    from oracle import engram as OE
    rng = np.random.default_rng(21)                           # same on every rank
    layer_ids, G, H, vocab = (1, 5), 4, 8, 2000
    primes, _ = OE.build_layout(len(layer_ids), G, H, vocab)
    sums = primes.reshape(len(layer_ids), -1).sum(-1)
    tm = rng.integers(0, 500, size=1200, dtype=np.int64)
    tm[7] = 499
    args = types.SimpleNamespace(engram_layer_ids=layer_ids,
                                 engram_num_embeddings=tuple(int(v) for v in sums),
                                 engram_max_ngram_size=G, engram_vocab_size=vocab,
                                 engram_n_heads=H, engram_pad_id=2,
                                 engram_compressed_vocab_size=500)
    h = engram.EngramHasher(args, tm, device=dev)
    rows, d, block = int(sums[1]), 512, 64
    table = torch.from_numpy(rng.integers(0, 126, size=(rows, d), dtype=np.uint8)).to(dev)
    scale = torch.from_numpy(rng.integers(115, 128, size=(rows, d // block),
                                          dtype=np.uint8)).to(dev)
    emb = engram.ParallelEngramEmbedding(rows, d, block)
    lo = emb.row_lo
    emb.weight = table[lo:lo + emb.part].contiguous()
    emb.scale = scale[lo:lo + emb.part].contiguous()
    full = engram.EngramEmbedding(rows, d, block)
    full.weight, full.scale = table, scale
    ids = torch.from_numpy(rng.integers(0, 1200, size=(2, 100), dtype=np.int64)).to(dev)
    ca = torch.zeros((2, 128), dtype=torch.int64, device=dev)
    cb = torch.zeros_like(ca)
    ok = True
    for s0, s1 in ((0, 5), (5, 37), (37, 100)):           # 10 and 64 positions fused, 126 not
        got = h.lookup_sum(emb, ids[:, s0:s1], s0, ca, layer=1)
        want = full.gather_sum(h(ids[:, s0:s1], s0, cb)[:, :, 1], torch.bfloat16)
        ok &= bool(torch.equal(got, want)) and bool(torch.equal(ca, cb))
    return ok


def _worker(rank, world, port, out_q):
    import datetime
    import sys
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401
    import importlib
    engram = importlib.import_module("deepseek_v41_mlx_b200.engram")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        rows, d, block = 20001, 1024, 32
        g = torch.Generator(device=dev).manual_seed(9)         # same table on every rank
        table = torch.randint(0, 126, (rows, d), dtype=torch.uint8, device=dev, generator=g)
        scale = torch.randint(115, 128, (rows, d // block), dtype=torch.uint8, device=dev,
                              generator=g)
        ok = True
        for T, H in ((300, 24), (1, 24), (5, 3)):
            idx = torch.randint(0, rows, (T, H), device=dev, generator=g)
            emb = engram.ParallelEngramEmbedding(rows, d, block)
            lo = emb.row_lo
            emb.weight = table[lo:lo + emb.part].contiguous()
            emb.scale = scale[lo:lo + emb.part].contiguous()
            full = engram.EngramEmbedding(rows, d, block)
            full.weight, full.scale = table, scale
            ok &= bool(torch.equal(emb.gather_sum(idx), full.gather_sum(idx, torch.bfloat16)))
            ok &= bool(torch.equal(emb(idx), full(idx, torch.bfloat16)))
        ok &= _lookup_sum_check(engram, dev)
        torch.cuda.synchronize()
        out_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_parallel_engram_matches_single_gpu():
    world = 2
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, qq)) for r in range(world)]
    for p in procs:
        p.start()
    res = [qq.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok in res:
        assert ok, f"rank {rank}: sharded lookup differs from the single table"
