"""Expert-parallel dispatch / combine bookkeeping on CPU with gloo (world size 2 and 3).

Each rank routes its own tokens, sends pairs to the experts' owners, the owners
apply their experts (a torch stand-in here; libdsv41q on GPUs), and the results
come back and are summed in top-k order.  The result must equal the
single-process computation of the same pairs exactly (same fp32 operations).
"""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, D, T, K = 12, 16, 7, 3



def _problem(seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(E, D, D, generator=g)
    xs = [torch.randn(T, D, generator=g) for _ in range(3)]
    idx = [torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]) for _ in range(3)]
    wts = [torch.rand(T, K, generator=g) for _ in range(3)]
    return W, xs, idx, wts


def _reference(W, x, idx, w):
    import importlib
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    Y = torch.stack([torch.stack([x[t] @ W[idx[t, j]].T for j in range(K)]) for t in range(T)])
    return ep.weighted_sum(Y, w)


def _worker(rank, world, init, out_q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401  (registers the package)
    import importlib
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        W, xs, idx, wts = _problem(0)
        epr = E // world
        x, ind, w = xs[rank], idx[rank], wts[rank]

        def experts(rows, local_ids):
            out = torch.empty(rows.shape[0], D)
            for i in range(rows.shape[0]):
                out[i] = rows[i] @ W[rank * epr + int(local_ids[i])].T
            return out

        rows, ids, order, sc, rc = ep.dispatch(dist, x, ind, world, epr)
        assert int(sum(rc)) == rows.shape[0] == ids.shape[0]
        assert all(0 <= int(i) < epr for i in ids)
        Y = ep.combine(dist, experts(rows, ids), order, sc, rc, T, K)
        got = ep.weighted_sum(Y, w)
        want = _reference(W, x, ind, w)
        out_q.put((rank, bool(torch.equal(got, want)), float((got - want).abs().max())))
    finally:
        dist.destroy_process_group()


def _prefill_reference(W, x, idx, w, shared):
    """Per pair bf16(w * (x W_e^T)), summed per token in ascending expert order, + shared."""
    Y = torch.stack([torch.stack([((x[t] @ W[idx[t, j]].T) * w[t, j]).to(torch.bfloat16)
                                  for j in range(K)]) for t in range(T)])
    import importlib
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    return ep.ascending_sum(Y, idx, shared)


def _prefill_worker(rank, world, init, out_q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401
    import importlib
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    dist.init_process_group("gloo", init_method=init, rank=rank, world_size=world)
    try:
        W, xs, idx, wts = _problem(1)
        epr = E // world
        x, ind, w = xs[rank], idx[rank], wts[rank]
        shared = torch.randn(T, D, generator=torch.Generator().manual_seed(7 + rank))

        def experts(rows, local_ids, recv_w):
            out = torch.empty(rows.shape[0], D, dtype=torch.bfloat16)
            for i in range(rows.shape[0]):
                out[i] = ((rows[i] @ W[rank * epr + int(local_ids[i])].T) * recv_w[i]).to(
                    torch.bfloat16)
            return out

        rows, ids, order, sc, rc, recv_w = ep.dispatch(dist, x, ind, world, epr, weights=w)
        assert recv_w.shape[0] == rows.shape[0]
        Y = ep.combine(dist, experts(rows, ids, recv_w), order, sc, rc, T, K)
        got = ep.ascending_sum(Y, ind, shared)
        want = _prefill_reference(W, x, ind, w, shared)
        out_q.put((rank, bool(torch.equal(got, want)), float((got - want).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ep_prefill_weights_travel_gloo(world, tmp_path):
    """Prefill form: routing weights travel with the pairs, outputs return as bf16 and are
    summed in ascending expert order -- exactly the single-process result."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = f"file://{tmp_path / 'rendezvous'}"   # no TCP port to race for
    procs = [ctx.Process(target=_prefill_worker, args=(r, world, init, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, err in res:
        assert same, f"rank {rank}: max err {err}"


def test_ascending_sum_order():
    import importlib
    import conftest  # noqa: F401
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    Y = torch.tensor([[[1.0], [1e8], [-1e8]]])          # fp32 order matters
    idx = torch.tensor([[7, 2, 5]])                      # ascending: 2, 5, 7
    got = ep.ascending_sum(Y, idx)
    assert float(got[0, 0]) == float((torch.tensor(0.0) + 1e8 - 1e8) + 1.0)


@pytest.mark.parametrize("world", [2, 3])
def test_ep_dispatch_combine_gloo(world, tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    init = f"file://{tmp_path / 'rendezvous'}"   # no TCP port to race for
    procs = [ctx.Process(target=_worker, args=(r, world, init, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, err in res:
        assert same, f"rank {rank}: max err {err}"


def test_plan_dispatch_orders_by_owner():
    import importlib
    import conftest  # noqa: F401
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    ind = torch.tensor([[5, 0, 11], [3, 7, 2]])
    order, counts = ep.plan_dispatch(ind, 3, 4)
    owners = (ind.reshape(-1) // 4)[order]
    assert torch.equal(owners, owners.sort().values)
    assert counts.tolist() == [3, 2, 1]        # owners 1,0,2,0,1,0
    # stable inside an owner: row-major pair order
    assert order.tolist()[:3] == [1, 3, 5]


@pytest.mark.parametrize("world", [2, 4])
def test_random_init_full_is_the_union_of_shards(world):
    """The single-GPU reference layer the bench checks expert parallelism against holds the
    same router, shared expert and experts as the ranks' shards together (CPU tensors)."""
    import deepseek_v41_mlx_b200 as q
    from deepseek_v41_mlx_b200.ep import EPMoE
    dev = torch.device("cpu")
    E, D, I, k = 8, 64, 32, 2
    full = EPMoE.random_init_full(q, torch, dev, world, E, D, I, k)
    epr = E // world
    for r in range(world):
        part = EPMoE.random_init(q, torch, dev, r, world, E, D, I, k)
        assert torch.equal(part.gate_w, full.gate.weight)
        assert torch.equal(part.gate_b, full.gate.bias)
        for name in ("gate_proj", "up_proj", "down_proj"):
            a, b = getattr(part.local.experts, name), getattr(full.experts, name)
            assert torch.equal(a.weight, b.weight[r * epr:(r + 1) * epr])
            assert torch.equal(a.scales, b.scales[r * epr:(r + 1) * epr])
        for key in ("w1", "w2", "w3"):
            a, b = getattr(part.local.shared_experts, key), getattr(full.shared_experts, key)
            assert torch.equal(a.weight, b.weight) and torch.equal(a.scales, b.scales)
