"""Row-sharded engram table (ParallelEngramEmbedding) on CPU with gloo, world size 2 and 3.

Every rank holds ceil(rows / world) rows; the indices are the same on every rank.  The
owners pack the raw rows each token slice needs, one all-to-all delivers them, the slice's
rank sums (or dequantizes) them, and an all-gather gives everyone the result.  The device
half is replaced by CPU functions with the kernels' arithmetic (fp32 products, adds in head
order), so the result must equal the single-process lookup of the whole table exactly.
"""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROWS, D, BLOCK = 50, 64, 32



def _table(world):
    """Codes avoid the e4m3 NaN bytes; pad rows (past ROWS) are zero codes, scale 1.0."""
    g = torch.Generator().manual_seed(3)
    part = -(-ROWS // world)
    codes = torch.randint(0, 126, (part * world, D), dtype=torch.uint8, generator=g)
    codes |= torch.randint(0, 2, (part * world, D), dtype=torch.uint8, generator=g) << 7
    scale = torch.randint(115, 128, (part * world, D // BLOCK), dtype=torch.uint8, generator=g)
    codes[ROWS:] = 0
    scale[ROWS:] = 127
    return codes, scale


def _dequant(codes, scale):
    v = codes.view(torch.float8_e4m3fn).float().reshape(codes.shape[0], -1, BLOCK)
    s = torch.ldexp(torch.ones(scale.shape), scale.to(torch.int32) - 127)
    return (v * s.unsqueeze(-1)).reshape(codes.shape[0], -1)


class CpuRowOps:
    def row_bytes(self, d, block):
        return (d + d // block + 15) // 16 * 16

    def pack_rows(self, weight, scale, row_lo, d, block, ids):
        out = torch.zeros(ids.numel(), self.row_bytes(d, block), dtype=torch.uint8)
        local = ids - row_lo
        ok = (local >= 0) & (local < weight.shape[0])
        out[ok, :d] = weight[local[ok]]
        out[ok, d:d + d // block] = scale[local[ok]]
        return out

    def _vals(self, recv, d, block):
        return _dequant(recv[:, :d].contiguous(), recv[:, d:d + d // block].contiguous())

    def sum_rows(self, recv, pos, d, block, out):
        vals = self._vals(recv, d, block)
        acc = torch.zeros(pos.shape[0], d)
        for h in range(pos.shape[1]):
            acc = acc + vals[pos[:, h]]
        out.copy_(acc.to(out.dtype))

    def dequant_rows(self, recv, pos, d, block, out):
        out.copy_(self._vals(recv, d, block)[pos].to(out.dtype))


def _reference_sum(codes, scale, idx):
    vals = _dequant(codes, scale)
    acc = torch.zeros(idx.shape[0], D)
    for h in range(idx.shape[1]):
        acc = acc + vals[idx[:, h]]
    return acc


def _cases(world):
    g = torch.Generator().manual_seed(7)
    part = -(-ROWS // world)
    return [torch.randint(0, ROWS, (7, 5), generator=g),          # ragged token slices
            torch.randint(0, ROWS, (1, 24), generator=g),          # fewer tokens than ranks
            torch.randint(0, part * world, (9, 3), generator=g)]   # ids in the pad rows too


def _worker(rank, world, init, out_q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401  (registers the package)
    import importlib
    engram = importlib.import_module("deepseek_v41_mlx_b200.engram")
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        codes, scale = _table(world)
        emb = engram.ParallelEngramEmbedding(ROWS, D, BLOCK, ops=CpuRowOps())
        assert (emb.rank, emb.world) == (rank, world)
        lo = emb.row_lo
        emb.weight, emb.scale = codes[lo:lo + emb.part].clone(), scale[lo:lo + emb.part].clone()
        results = []
        for idx in _cases(world):
            s = emb.gather_sum(idx, out_dtype=torch.float32)
            r = emb(idx, out_dtype=torch.float32)
            results.append((s, r))
        # numpy copies travel by plain pickling: a torch tensor put on the queue goes through a
        # shared-memory handle that can vanish when this process exits before it is read
        out_q.put((rank, [(s.numpy().copy(), r.numpy().copy()) for s, r in results], None))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_parallel_engram_matches_single_table(world, tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = f"file://{tmp_path / 'rendezvous'}"   # no TCP port to race for
    procs = [ctx.Process(target=_worker, args=(r, world, init, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        rank, res, err = q.get(timeout=180)
        assert err is None, f"rank {rank}: {err}"
        got[rank] = res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    codes, scale = _table(world)
    for ci, idx in enumerate(_cases(world)):
        want_sum = _reference_sum(codes, scale, idx)
        want_rows = _dequant(codes, scale)[idx.reshape(-1)].reshape(tuple(idx.shape) + (D,))
        for rank in range(world):
            s, r = (torch.from_numpy(a) for a in got[rank][ci])
            assert torch.equal(s, want_sum), f"case {ci} rank {rank}: summed rows differ"
            assert torch.equal(r, want_rows), f"case {ci} rank {rank}: rows differ"


def test_plan_is_consistent_across_ranks():
    """What each owner sends to a rank is exactly what that rank expects, in order."""
    import importlib
    engram = importlib.import_module("deepseek_v41_mlx_b200.engram")
    g = torch.Generator().manual_seed(11)
    for world in (2, 3, 4):
        idx = torch.randint(0, ROWS, (10, 6), generator=g)
        plans = [engram.ParallelEngramEmbedding(ROWS, D, BLOCK, rank=r, world=world,
                                                ops=CpuRowOps()).plan(idx)
                 for r in range(world)]
        for r in range(world):
            assert plans[r]["recv_counts"] == [plans[o]["send_counts"][r] for o in range(world)]
            # rows rank r receives, in buffer order, must be the ids its positions name
            recv_ids = []
            for o in range(world):
                sc = plans[o]["send_counts"]
                start = sum(sc[:r])
                recv_ids.append(plans[o]["send_ids"][start:start + sc[r]])
            recv_ids = torch.cat(recv_ids)
            t0, t1 = plans[r]["t0"], plans[r]["t1"]
            assert torch.equal(recv_ids[plans[r]["recv_pos"]], idx[t0:t1])
