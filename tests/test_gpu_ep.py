"""Expert-parallel MoE prefill on 2 GPUs (NCCL) vs the single-GPU layer.

Each rank routes its own tokens (given routing), sends the pairs to the experts' owners
with their routing weights, gets bf16 expert outputs back and sums them in ascending
expert order before adding the shared expert.  The single-GPU reference holds all experts
(gathered from the ranks) and runs the same kernels on the same tokens: the per-row results
do not depend on which other rows share a GEMM tile, so the outputs are identical bits.
Skipped with fewer than 2 GPUs; run with a 2-GPU box.
"""

from __future__ import annotations

import ctypes
import os
import socket
import types

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


def _worker(rank, world, port, out_q):
    import datetime
    import sys
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401
    import importlib
    q = importlib.import_module("deepseek_v41_mlx_b200")
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        E, D, I, k, T = 8, 256, 256, 3, 96
        layer = ep.EPMoE.random_init(q, torch, dev, rank, world, E, D, I, k, seed=3)
        g = torch.Generator(device=dev).manual_seed(100 + rank)
        x = torch.randn(T, D, generator=g, device=dev).to(torch.bfloat16)
        idx = torch.stack([torch.randperm(E, generator=g, device=dev)[:k] for _ in range(T)])
        idx = idx.to(torch.int32)
        w = torch.rand(T, k, generator=g, device=dev) + 0.1
        y = layer.forward_prefill(x, weights=w, indices=idx, out_dtype=torch.float32)
        # the single-GPU layer with every expert
        args = types.SimpleNamespace(n_activated_experts=k, score_func="sqrtsoftplus",
                                     gate_temp=1.0, norm_topk_prob=True, route_scale=1.5,
                                     n_routed_experts=E, dim=D, moe_inter_dim=I,
                                     swiglu_limit=10.0)
        full = q.moe.MoE(args, round_bf16=True, cuda_graph=False)
        full.gate.weight, full.gate.bias = layer.gate_w, layer.gate_b
        for name in ("gate_proj", "up_proj", "down_proj"):
            src = getattr(layer.local.experts, name)
            for attr in ("weight", "scales"):
                part = getattr(src, attr).contiguous()
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                setattr(getattr(full.experts, name), attr, torch.cat(parts, 0))
        for key in ("w1", "w2", "w3"):
            s = getattr(layer.local.shared_experts, key)
            setattr(getattr(full.shared_experts, key), "weight", s.weight)
            setattr(getattr(full.shared_experts, key), "scales", s.scales)
        y_full = full.prefill_a8(x, weights=w, indices=idx, out_dtype=torch.float32)
        torch.cuda.synchronize()
        out_q.put((rank, bool(torch.equal(y, y_full)), float((y - y_full).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_prefill_matches_single_gpu():
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
    for rank, same, err in res:
        assert same, f"rank {rank}: max abs diff {err}"


def _decode_worker(rank, world, port, out_q):
    import datetime
    import sys
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    import conftest  # noqa: F401
    import importlib
    q = importlib.import_module("deepseek_v41_mlx_b200")
    ep = importlib.import_module("deepseek_v41_mlx_b200.ep")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        E, D, I, k = 16, 512, 256, 4
        layer = ep.EPMoE.random_init(q, torch, dev, rank, world, E, D, I, k, seed=5)
        layer.max_tokens = 48
        args = types.SimpleNamespace(n_activated_experts=k, score_func="sqrtsoftplus",
                                     gate_temp=1.0, norm_topk_prob=True, route_scale=1.5,
                                     n_routed_experts=E, dim=D, moe_inter_dim=I,
                                     swiglu_limit=10.0)
        full = q.moe.MoE(args, round_bf16=True, cuda_graph=False)
        full.gate.weight, full.gate.bias = layer.gate_w, layer.gate_b
        for name in ("gate_proj", "up_proj", "down_proj"):
            src = getattr(layer.local.experts, name)
            for attr in ("weight", "scales"):
                part = getattr(src, attr).contiguous()
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                setattr(getattr(full.experts, name), attr, torch.cat(parts, 0))
        for key in ("w1", "w2", "w3"):
            s = getattr(layer.local.shared_experts, key)
            setattr(getattr(full.shared_experts, key), "weight", s.weight)
            setattr(getattr(full.shared_experts, key), "scales", s.scales)
        g = torch.Generator(device=dev).manual_seed(200 + rank)
        # several steps, a different token count per rank and step (0 = this rank idles)
        counts = [(5, 33), (1, 48), (0, 7), (17, 2)]
        same = True
        worst = 0.0
        for step, tc in enumerate(counts):
            T = tc[rank]
            x = torch.randn(T, D, generator=g, device=dev).to(torch.bfloat16)
            y, w, idx = layer.forward(x, with_routing=True)
            if T:
                yf, wf, idxf = full(x, with_routing=True)
                torch.cuda.synchronize()
                ok = (torch.equal(y, yf) and torch.equal(w, wf) and torch.equal(idx, idxf))
                same &= bool(ok)
                worst = max(worst, float((y.float() - yf.float()).abs().max()))
        torch.cuda.synchronize()
        layer.close()
        flags = ctypes.c_uint32(0)
        q._lib.call("dsv41_device_status", torch.cuda.current_stream().cuda_stream,
                    ctypes.byref(flags))
        out_q.put((rank, same, worst, int(flags.value)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_decode_peer_memory_matches_single_gpu():
    """Decode with the pairs sent to their owners and back through NVLink peer stores gives
    the single-GPU layer's bits (outputs, routing weights, indices) on every step."""
    world = 2
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decode_worker, args=(r, world, port, qq)) for r in range(world)]
    for p in procs:
        p.start()
    res = [qq.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, same, worst, flags in res:
        assert flags == 0, f"rank {rank}: device status {flags} (a bounded wait expired)"
        assert same, f"rank {rank}: max abs diff {worst}"
