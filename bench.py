"""Benchmark of the quantized-weight MoE decode layer.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one MoE-layer forward at decode (router + fp4 routed experts + fp8
shared expert + combine) over one batch of T=64 tokens of synthetic bf16
activations, with random-init weights of the release layout: 384 experts,
dim 7168, moe_inter_dim 2048, top-6, ue8m0 scales in [120, 128].  The headline
`value` is whole-job tokens/s with inputs resident in HBM; `e2e` is the same
step through the public API with pinned host input/output buffers copied inside
the timed region.  Sub-measurements (T=1, T=8, the fp8 dense GEMV, the MLX
affine GEMV and the engram gather) are reported under "sub".

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize(); each step is timed with CUDA events on the launching
stream; L2 is flushed (256 MiB write) between steps outside the events and the
input batch rotates over 8 pre-generated batches.  Multi-GPU: one process per
GPU (torchrun), each rank serves its own batch with the experts sharded
expert-parallel over NCCL all-to-all (see deepseek-v41-mlx_b200/ep.py); the
reported time is the max over ranks.

--impl reference times the reference's CPU implementation of this path (the
numpy oracle restating deepseek_v41_mlx/moe.py + dequant.py; the MLX original
cannot be installed offline) on the host cores, on a bounded sample of the same
workload, and prints the same JSON line with "impl": "reference".
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "deepseek-v41-mlx_b200")
METRIC = "MoE-layer tok/s at batch 1/64/8192; dequant-GEMV HBM GB/s vs 8 TB/s"
E, D, I, TOPK = 384, 7168, 2048, 6
T_HEAD = 64
BYTES_PER_EXPERT = 3 * (I * D // 2 + I * D // 32)        # 23,396,352 (fp4 + ue8m0)
GU_BYTES_PER_EXPERT = 2 * (I * D // 2 + I * D // 32)     # gate + up
ROUTER_BYTES = E * D * 2
SHARED_BYTES = 3 * (I * D + (I // 32) * (D // 32))


def _package():
    name = "deepseek_v41_mlx_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------- clocks sampler --

class Clocks:
    """nvidia-smi sampled every 200 ms while the timed region runs."""

    def __init__(self, index=0):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.3)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        busy = [v for v in sm if v > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- setup --

def make_moe(q, torch, device, seed=0, n_local=None):
    """Random-init weights of the release layout, generated on the device."""
    import types
    n_local = E if n_local is None else n_local
    g = torch.Generator(device=device).manual_seed(seed)
    args = types.SimpleNamespace(n_activated_experts=TOPK, score_func="sqrtsoftplus", gate_temp=1.0,
                                 norm_topk_prob=True, route_scale=1.5, n_routed_experts=E, dim=D,
                                 moe_inter_dim=I, swiglu_limit=10.0)
    m = q.moe.MoE(args, round_bf16=True)
    m.gate.weight = (torch.randn(E, D, device=device, generator=g) * D ** -0.5).to(torch.bfloat16)
    m.gate.bias = torch.randn(E, device=device, generator=g) * 0.01
    for name, (n, k) in (("gate_proj", (I, D)), ("up_proj", (I, D)), ("down_proj", (D, I))):
        pr = getattr(m.experts, name)
        pr.weight = torch.randint(0, 256, (n_local, n, k // 2), dtype=torch.uint8, device=device,
                                  generator=g)
        pr.scales = torch.randint(120, 129, (n_local, n, k // 32), dtype=torch.uint8,
                                  device=device, generator=g)
    for key, (n, k) in (("1", (I, D)), ("3", (I, D)), ("2", (D, I))):
        w = torch.randint(0, 256, (n, k), dtype=torch.uint8, device=device, generator=g)
        w[(w & 0x7F) == 0x7F] = 0
        pr = getattr(m.shared_experts, "w" + key)
        pr.weight = w
        pr.scales = torch.randint(118, 128, (n // 32, k // 32), dtype=torch.uint8, device=device,
                                  generator=g)
    return m


def zipf_routing(torch, dev, x, gate_w, T, seed=7, s=1.1):
    """BASELINE.json configs[2] routing: per token, top-6 expert ids drawn without
    replacement from Zipf(s) over a seeded permutation of the experts (Gumbel-top-k on
    log p_zipf); weights = the router's unbiased sqrt-softplus scores at those ids,
    normalised and scaled by route_scale 1.5."""
    g = torch.Generator(device=dev).manual_seed(seed)
    perm = torch.randperm(E, device=dev, generator=g)
    logp = torch.empty(E, device=dev)
    logp[perm] = -s * torch.log(torch.arange(1, E + 1, device=dev, dtype=torch.float32))
    u = torch.rand(T, E, device=dev, generator=g).clamp_(1e-30, 1.0)
    idx = (logp[None, :] - torch.log(-torch.log(u))).topk(TOPK, dim=-1).indices
    scores = torch.sqrt(torch.nn.functional.softplus(x.float() @ gate_w.float().T))
    w = scores.gather(1, idx)
    w = w / (w.sum(-1, keepdim=True) + 1e-20) * 1.5
    return w.contiguous(), idx.to(torch.int32).contiguous()


def prefill_measurement(q, torch, dev, layer, flush, stream, peaks, K, W, T=8192):
    """d3: the layer at prefill in a8 numerics (upstream linear()), T=8192, Zipf routing."""
    hbm_peak, bf16_peak, peak_src = peaks
    g = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = zipf_routing(torch, dev, x, layer.gate.weight, T)
    counts = torch.bincount(idx.reshape(-1).long(), minlength=E)
    fn = lambda i: layer.prefill_a8(x, weights=w, indices=idx)
    ms = timed_steps(torch, fn, K, W, flush, stream)
    st = statistics.median(ms)
    q._lib.prof_enable(True)
    fn(0)
    torch.cuda.synchronize()
    prof = q._lib.prof_report()
    q._lib.prof_enable(False)
    f_routed = 2.0 * T * TOPK * 3 * I * D
    f_shared = 2.0 * 3 * T * I * D
    fp8_peak = 2.0 * bf16_peak          # f8f6f4 rate = twice the bf16 rate
    kern = {k: round(v[1] / v[0], 4) for k, v in prof.items()}
    gu, dn = kern.get("pf_gate_up_fp4"), kern.get("pf_down_fp4")
    routed_ms = (gu or 0) + (dn or 0)
    active = int((counts > 0).sum())
    wbytes = active * BYTES_PER_EXPERT
    return {
        "tok_s": round(T / (st / 1e3), 1), "ms": round(st, 4), "tokens": T,
        "tflops_layer": round((f_routed + f_shared) / (st / 1e3) / 1e12, 1),
        "routed_gemm_tflops": round(f_routed / (routed_ms / 1e3) / 1e12, 1) if routed_ms else None,
        "routed_gemm_frac_fp8_peak": round(f_routed / (routed_ms / 1e3) / 1e12 / fp8_peak, 4)
        if routed_ms else None,
        "routed_weight_gbs": round(wbytes / (routed_ms / 1e3) / 1e9, 1) if routed_ms else None,
        "fp8_peak_tflops": fp8_peak, "peak_source": peak_src + " 2x bf16_tflops",
        "kernel_ms": kern, "experts_active": active, "pairs_max_expert": int(counts.max()),
        "pairs_min_expert": int(counts.min()),
        "routing": "Zipf(1.1) Gumbel-top-6 over a seeded expert permutation; router-score weights",
    }


def timed_steps(torch, fn, K, W, flush, stream):
    """W warm-up calls, then K calls each between CUDA events; returns per-step ms."""
    for i in range(W):
        fn(i)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(K)]
    for i in range(K):
        flush.zero_()
        ev[i][0].record(stream)
        fn(W + i)
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


# ---------------------------------------------------------------- our arm --

def run_ours(args):
    import torch
    import torch.distributed as dist
    q = _package()
    q._lib.load()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    hbm_peak, bf16_peak, peak_src = _peaks()
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)

    if world > 1:
        from importlib import import_module
        ep = import_module("deepseek_v41_mlx_b200.ep")
        layer = ep.EPMoE.random_init(q, torch, dev, rank, world, E, D, I, TOPK)
        fwd = layer.forward
    else:
        layer = make_moe(q, torch, dev)
        # the headline replays CUDA graphs captured from the layer's launches (one graph per
        # timed step): the library's launch-timing events around the dominant kernel are
        # event nodes of each graph, so its duration is measured inside the timed region
        layer.cuda_graph = False
        fwd = layer

    def batches(T, n=8):
        return [torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(n)]

    xs = batches(T_HEAD)
    K, W = args.steps, args.warmup

    # ---- headline: T = 64, device-resident inputs, launch timing enabled ----
    q._lib.prof_enable(False)
    for i in range(W):
        fwd(xs[i % len(xs)])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    q._lib.prof_enable(True)
    q._lib.prof_select(["moe_expert_gate_up_fp4"])   # events around the dominant kernel only
    if world == 1:
        steps = []
        for i in range(K):                            # one graph per timed step
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fwd(xs[i % len(xs)])
            steps.append(gr)
        launches = q._lib.prof_launches()             # counted once per captured launch
        for i in range(W):
            steps[i % K].replay()
        step_fn = lambda i: steps[i].replay()
    else:
        step_fn = lambda i: fwd(xs[i % len(xs)])
    with Clocks(local) as clk:
        ms = timed_steps(torch, step_fn, K, 0, flush, stream)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    prof = q._lib.prof_report()
    if world > 1:
        launches = q._lib.prof_launches()
    else:
        del steps
    q._lib.prof_select(None)
    q._lib.prof_enable(False)
    # per-kernel breakdown (every kernel bracketed by events): a separate, untimed pass
    q._lib.prof_enable(True)
    timed_steps(torch, lambda i: fwd(xs[i % len(xs)]), max(3, K // 4), 0, flush, stream)
    kprof = q._lib.prof_report()
    q._lib.prof_enable(False)
    step_ms = sum(ms) / len(ms)
    if world > 1:
        t = torch.tensor([step_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = float(t.item())
    value = T_HEAD * world / (step_ms / 1e3)

    # active experts per step (for the algorithmic byte count), outside timing
    active = []
    if world > 1:
        layer.track = True                       # this rank's local experts per step
        for x in xs[:4]:
            layer.forward(x)                     # collective: every rank runs the same count
        layer.track = False
    for x in xs[:4]:
        _, _, idx = (layer.full_routing(x) if world > 1 else fwd(x, with_routing=True))
        active.append(len(torch.unique(idx)))
    n_act = statistics.mean(active)

    gu = prof.get("moe_expert_gate_up_fp4")
    roof = None
    if gu:
        gu_ms = gu[1] / gu[0]
        n_act_local = n_act if world == 1 else n_act  # per-rank local experts (EP) below
        if world > 1:
            n_act_local = layer.local_active_mean
        gu_bytes = n_act_local * GU_BYTES_PER_EXPERT
        achieved = gu_bytes / (gu_ms / 1e3) / 1e9
        traffic = None
        tf = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tf):
            tr = json.load(open(tf)).get("moe_expert_gate_up_fp4")
            if tr:
                traffic = tr["dram_bytes_per_active_expert"] * n_act_local
        roof = {"bound": "hbm", "kernel": "moe_expert_gate_up_fp4", "achieved": round(achieved, 1),
                "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                "traffic": traffic, "algorithmic_bytes": int(gu_bytes),
                "avg_launch_ms": round(gu_ms, 5), "peak_source": peak_src + " hbm_gbs (copy)"}
    layer_bytes = n_act * BYTES_PER_EXPERT + ROUTER_BYTES + SHARED_BYTES
    layer_gbs = layer_bytes / (step_ms / 1e3) / 1e9 if world == 1 else None

    # ---- e2e: pinned host buffers, copies inside the timed region ----
    xh = [x.cpu().pin_memory() for x in xs]
    yh = torch.empty((T_HEAD, D), dtype=torch.bfloat16).pin_memory()
    xd = torch.empty((T_HEAD, D), dtype=torch.bfloat16, device=dev)

    if world == 1:
        layer.cuda_graph = True      # the public API's default: the layer replays its own graph

    def e2e_step(i):
        xd.copy_(xh[i % len(xh)], non_blocking=True)
        y = fwd(xd)
        yh.copy_(y, non_blocking=True)

    ms_e2e = timed_steps(torch, e2e_step, K, W, flush, stream)
    e2e_ms = sum(ms_e2e) / len(ms_e2e)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(T_HEAD * world / (e2e_ms / 1e3), 1), "unit": "tok/s",
           "h2d_bytes_per_step": T_HEAD * D * 2, "d2h_bytes_per_step": T_HEAD * D * 2}

    sub = {}
    if world == 1 and not args.no_sub:
        sub = sub_measurements(q, torch, dev, layer, flush, stream, hbm_peak, max(3, K // 2), W)
        sub["moe_prefill_T8192_a8"] = prefill_measurement(
            q, torch, dev, layer, flush, stream, (hbm_peak, bf16_peak, peak_src), max(3, K // 4), W)
        sub.update(engram_measurement(q, torch, dev, flush, stream, max(3, K // 2), W))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(seconds=args.cpu_seconds)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp4-e2m1 weights x bf16 act (f16 mma, f32 acc)",
        "data": "synthetic (random-init weights of the release layout, N(0,1) bf16 activations)",
        "config": {"workload": "moe_decode_fp4 (BASELINE.json configs[1]) at T=64",
                   "experts": E, "dim": D, "moe_inter_dim": I, "topk": TOPK, "tokens_per_gpu": T_HEAD,
                   "global_batch": T_HEAD * world,
                   "parallelism": "ep%d" % world if world > 1 else "single",
                   "l2": "flushed (256 MiB write) between timed steps; inputs rotate over 8 batches",
                   "active_experts_mean": round(n_act, 1),
                   "layer_bytes_per_step": int(layer_bytes)},
        "roofline": roof,
        "layer_hbm_gbs": round(layer_gbs, 1) if layer_gbs else None,
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
        "kernel_ms": {k: round(v[1] / v[0], 5) for k, v in kprof.items()},
        "clocks": clk.summary(), "sub": sub,
    }
    print(json.dumps(line))


def graphed(torch, fns):
    """Capture each call (through the public API) into a CUDA graph, after one warm-up."""
    out = []
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(side)
    for f in fns:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            f()
        out.append(g)
    return out


def sub_measurements(q, torch, dev, layer, flush, stream, hbm_peak, K, W):
    out = {}
    g = torch.Generator(device=dev).manual_seed(99)
    layer.cuda_graph = True
    for T in (1, 8, 64):
        xs = [torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(8)]
        ms = timed_steps(torch, lambda i: layer(xs[i % 8]), K, W, flush, stream)
        act = statistics.mean(len(torch.unique(layer(x, with_routing=True)[2])) for x in xs[:4])
        st = sum(ms) / len(ms)
        byts = act * BYTES_PER_EXPERT + ROUTER_BYTES + SHARED_BYTES
        out[f"moe_decode_T{T}_graph"] = {"tok_s": round(T / (st / 1e3), 1), "ms": round(st, 4),
                                         "layer_gbs": round(byts / (st / 1e3) / 1e9, 1),
                                         "frac_hbm": round(byts / (st / 1e3) / 1e9 / hbm_peak, 4)}
    layer.cuda_graph = False
    # d1: fp8 dense [4096, 7168], several weight copies (> 4x L2) rotated
    N, Kd = 4096, 7168
    copies = 10
    ws = [torch.randint(0, 256, (N, Kd), dtype=torch.uint8, device=dev, generator=g)
          for _ in range(copies)]
    ss = [torch.randint(118, 128, (N // 32, Kd // 32), dtype=torch.uint8, device=dev, generator=g)
          for _ in range(copies)]
    for w in ws:
        w[(w & 0x7F) == 0x7F] = 0
    for M in (1, 32):
        x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
        gr = graphed(torch, [lambda c=c: q.linear.linear_fp8(x, ws[c], ss[c]) for c in range(copies)])
        ms = timed_steps(torch, lambda i: gr[i % copies].replay(), K * 4, W, flush, stream)
        st = sum(ms) / len(ms)
        byts = N * Kd + (N // 32) * (Kd // 32) + M * Kd * 2 + M * N * 2
        # the same GEMV over the 10 weight copies back to back in one graph (a decode step
        # runs many such products in a row): time per GEMV
        chain = graphed(torch, [lambda: [q.linear.linear_fp8(x, ws[c], ss[c]) for c in range(copies)]])[0]
        msc = timed_steps(torch, lambda i: chain.replay(), K, W, flush, stream)
        stc = sum(msc) / len(msc) / copies
        out[f"gemv_fp8_block_M{M}"] = {"ms": round(st, 5), "gbs": round(byts / st / 1e6, 1),
                                       "frac_hbm": round(byts / st / 1e6 / hbm_peak, 4),
                                       "chained_ms": round(stc, 5),
                                       "chained_gbs": round(byts / stc / 1e6, 1),
                                       "chained_frac_hbm": round(byts / stc / 1e6 / hbm_peak, 4)}
    del ws, ss
    out.update(affine_prefill_measurement(q, torch, dev, flush, stream, K, W))
    # d4: MLX affine [14336, 7168], 4 and 8 bit
    N, Kd = 14336, 7168
    for bits in (4, 8):
        copies = 4 if bits == 4 else 3
        wq = [torch.randint(-2 ** 31, 2 ** 31 - 1, (N, Kd * bits // 32), dtype=torch.int32,
                            device=dev, generator=g) for _ in range(copies)]
        sc = [(torch.rand(N, Kd // 64, device=dev, generator=g) * 0.019 + 0.001).to(torch.bfloat16)
              for _ in range(copies)]
        bi = [(torch.randn(N, Kd // 64, device=dev, generator=g) * 0.05).to(torch.bfloat16)
              for _ in range(copies)]
        for M in (1, 16):
            x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
            gr = graphed(torch, [lambda c=c: q.linear.linear_affine(x, wq[c], sc[c], bi[c], bits)
                                 for c in range(copies)])
            ms = timed_steps(torch, lambda i: gr[i % copies].replay(), K * 4, W, flush, stream)
            st = sum(ms) / len(ms)
            byts = N * Kd * bits // 8 + 2 * N * (Kd // 64) * 2 + M * Kd * 2 + M * N * 2
            out[f"gemv_affine{bits}_M{M}"] = {"ms": round(st, 5), "gbs": round(byts / st / 1e6, 1),
                                              "frac_hbm": round(byts / st / 1e6 / hbm_peak, 4)}
        del wq, sc, bi
    # converter (next row 3): mx.quantize of a bf16 [14336, 7168] weight, groups of 64; two
    # weight copies (> L2) rotated; bytes = bf16 in + codes + bf16 scales and biases out
    ws_bf = [torch.randn(N, Kd, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
    for bits in (4, 8):
        gr = graphed(torch, [lambda c=c: q.dequant.quantize_affine(ws_bf[c], 64, bits)
                             for c in range(2)])
        ms = timed_steps(torch, lambda i: gr[i % 2].replay(), K * 2, W, flush, stream)
        st = sum(ms) / len(ms)
        byts = N * Kd * 2 + N * Kd * bits // 8 + 2 * N * (Kd // 64) * 2
        out[f"quantize_affine{bits}_14336x7168"] = {
            "ms": round(st, 4), "gbs": round(byts / st / 1e6, 1),
            "frac_hbm": round(byts / st / 1e6 / hbm_peak, 4)}
        del gr
    del ws_bf
    return out


def affine_prefill_measurement(q, torch, dev, flush, stream, K, W, M=4096):
    """d4 at prefill: MLX affine [14336, 7168] 4- and 8-bit, M = 4096 activation rows, on the
    tensor cores (weights dequantized to bf16 per tile); TFLOP/s against the bf16 peak."""
    _, bf16_peak, peak_src = _peaks()
    N, Kd = 14336, 7168
    g = torch.Generator(device=dev).manual_seed(77)
    x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
    out = {}
    for bits in (4, 8):
        wq = torch.randint(-2 ** 31, 2 ** 31 - 1, (N, Kd * bits // 32), dtype=torch.int32,
                           device=dev, generator=g)
        sc = (torch.rand(N, Kd // 64, device=dev, generator=g) * 0.019 + 0.001).to(torch.bfloat16)
        bi = (torch.randn(N, Kd // 64, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        ms = statistics.median(timed_steps(
            torch, lambda i: q.linear.linear_affine(x, wq, sc, bi, bits), K, W, flush, stream))
        tf = 2.0 * M * N * Kd / (ms / 1e3) / 1e12
        out[f"qmm_affine{bits}_M{M}"] = {"ms": round(ms, 4), "tflops": round(tf, 1),
                                         "frac_bf16_peak": round(tf / bf16_peak, 4),
                                         "peak_source": peak_src + " bf16_tflops"}
        del wq, sc, bi
    return out


def engram_measurement(q, torch, dev, flush, stream, K, W, vocab=4_000_000):
    """d5: engram table fp8 e4m3 [96,000,xxx x 1024] (one ue8m0 per row, [115, 127]) built on
    the device, 24 rows per token (2/3/4-gram x 8 heads, one layer, primes from 4,000,000)
    hashed from uniform compressed ids in [0, 99092); a step = hash + gather + dequant + fp32
    sum -> bf16 [T, 1024] through EngramHasher.lookup_sum (one launch at T=1, the hasher then
    the gather-sum above its fused_max_positions); ``ms_two_step`` always times the latter.  Bytes per token: 24 x (1024 + 1) read + 2048 written.  A smaller
    ``vocab`` (engram_vocab_size) gives a table of about 24 x vocab rows, for ncu captures."""
    import types
    import numpy as np
    hbm_peak, _, peak_src = _peaks()
    args = types.SimpleNamespace(engram_layer_ids=(1,), engram_max_ngram_size=4,
                                 engram_vocab_size=vocab, engram_n_heads=8, engram_pad_id=2,
                                 engram_compressed_vocab_size=99092)
    primes, _ = q.engram.build_layout(args)
    rows, d = int(primes.sum()), 1024
    args.engram_num_embeddings = (rows,)
    hasher = q.engram.EngramHasher(args, np.arange(99092, dtype=np.int64), device=dev)
    g = torch.Generator(device=dev).manual_seed(55)
    # the table stored packed (EngramEmbedding.pack: codes then the row's scale, 1040 bytes a
    # row), generated in place: uniform over non-NaN codes, scales in [115, 127]
    rb = int(q._lib.load().dsv41_engram_row_bytes(d, d))
    table = torch.zeros((rows, rb), dtype=torch.uint8, device=dev)
    for r0 in range(0, rows, 1 << 20):          # 1 GB at a time
        c = table[r0:r0 + (1 << 20), :d]
        c.random_(0, 254, generator=g)
        c += (c >= 127).to(torch.uint8)
        table[r0:r0 + (1 << 20), d].random_(115, 128, generator=g)
    emb = q.engram.EngramEmbedding(rows, d, block=d)
    emb.packed = table
    out = {}
    for T in (1, 8192):
        start = 100 if T == 1 else 0
        ids = [torch.randint(0, 99092, (1, T), dtype=torch.int64, device=dev, generator=g)
               for _ in range(8)]
        cache = torch.randint(0, 99092, (1, start + T + 8), dtype=torch.int64, device=dev,
                              generator=g)

        def step(i, T=T, start=start):
            # hash + gather-sum (one launch up to EngramHasher.fused_max_positions positions)
            return hasher.lookup_sum(emb, ids[i % 8], start, cache)

        def step2(i, T=T, start=start):
            idx = hasher(ids[i % 8], start, cache)
            return emb.gather_sum(idx.reshape(T, -1))

        # the step replayed from CUDA graphs (one per input batch): device time, no host gaps
        gr = graphed(torch, [lambda c=c: step(c) for c in range(8)])
        ms = statistics.median(timed_steps(torch, lambda i: gr[i % 8].replay(), K, W, flush,
                                           stream))
        ms_host = statistics.median(timed_steps(torch, step, K, W, flush, stream))
        gr2 = graphed(torch, [lambda c=c: step2(c) for c in range(8)])
        ms2 = statistics.median(timed_steps(torch, lambda i: gr2[i % 8].replay(), K, W, flush,
                                            stream))
        del gr2
        byts = T * (24 * (d + 1) + 2 * d)
        out[f"engram_T{T}"] = {"ms": round(ms, 4), "ms_eager": round(ms_host, 4),
                               "ms_two_step": round(ms2, 4),
                               "tok_s": round(T / (ms / 1e3), 1),
                               "gbs": round(byts / (ms / 1e3) / 1e9, 1),
                               "frac_hbm": round(byts / (ms / 1e3) / 1e9 / hbm_peak, 4),
                               "table_rows": rows, "table_gb": round(rows * rb / 1e9, 1),
                               "table_layout": "packed rows (codes + scale, %d B)" % rb,
                               "peak_source": peak_src + " hbm_gbs"}
    del table, emb
    torch.cuda.empty_cache()
    return out


def run_prefill_ep(args):
    """d3 over NCCL: each rank prefills its own T tokens (weak scaling) with E / ws experts;
    the step is timed with CUDA events per rank, max over ranks."""
    import datetime
    import torch
    import torch.distributed as dist
    from importlib import import_module
    q = _package()
    ep = import_module("deepseek_v41_mlx_b200.ep")
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    T = args.prefill_tokens
    layer = ep.EPMoE.random_init(q, torch, dev, rank, world, E, D, I, TOPK)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = zipf_routing(torch, dev, x, layer.gate_w, T, seed=7 + rank)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    fn = lambda i: layer.forward_prefill(x, weights=w, indices=idx)
    for i in range(args.warmup):
        fn(i)
    torch.cuda.synchronize()
    dist.barrier()
    with Clocks(local) as clk:
        ms = timed_steps(torch, fn, args.steps, 0, flush, stream)
        dist.barrier()
        torch.cuda.synchronize()
    st = torch.tensor([statistics.median(ms)], device=dev)
    dist.all_reduce(st, op=dist.ReduceOp.MAX)
    layer.track = True
    fn(0)
    layer.track = False
    loc = torch.tensor([float(layer.local_active[-1])], device=dev)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        step = float(st.item())
        print(json.dumps({"metric": "MoE-layer prefill tok/s (a8, EP)", "tok_s": round(T * world / (step / 1e3), 1),
                          "ms": round(step, 4), "n_gpus": world, "tokens_per_gpu": T,
                          "parallelism": "ep%d" % world, "experts_per_gpu": E // world,
                          "scaling": "weak", "clocks": clk.summary(),
                          "routing": "Zipf(1.1) per rank (seed 7 + rank)"}))


def run_engram_ep(args):
    """d5 row-sharded over NCCL (upstream ParallelEngramEmbedding layout): rank r holds rows
    [r * part, (r + 1) * part) of the 96M-row table; every rank hashes the same T tokens (the
    tensor-parallel setting upstream runs in), the owners send the raw rows each token slice
    needs (one all-to-all), slices are summed in head order and all-gathered.  Total work is
    fixed as ranks are added ("strong"); a step is timed with CUDA events per rank, max over
    ranks."""
    import datetime
    import types
    import numpy as np
    import torch
    import torch.distributed as dist
    q = _package()
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
    hbm_peak, _, peak_src = _peaks()
    eargs = types.SimpleNamespace(engram_layer_ids=(1,), engram_max_ngram_size=4,
                                  engram_vocab_size=4_000_000, engram_n_heads=8, engram_pad_id=2,
                                  engram_compressed_vocab_size=99092)
    primes, _ = q.engram.build_layout(eargs)
    rows, d = int(primes.sum()), 1024
    eargs.engram_num_embeddings = (rows,)
    hasher = q.engram.EngramHasher(eargs, np.arange(99092, dtype=np.int64), device=dev)
    emb = q.engram.ParallelEngramEmbedding(rows, d, block=d)
    g = torch.Generator(device=dev).manual_seed(55 + rank)
    table = torch.empty((emb.part, d), dtype=torch.uint8, device=dev)
    for r0 in range(0, emb.part, 1 << 20):
        c = table[r0:r0 + (1 << 20)]
        c.random_(0, 254, generator=g)
        c += (c >= 127).to(torch.uint8)
    emb.weight = table
    emb.scale = torch.randint(115, 128, (emb.part, 1), dtype=torch.uint8, device=dev, generator=g)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    res = {}
    gi = torch.Generator(device=dev).manual_seed(77)          # same ids on every rank
    for T in (1, 8192):
        start = 100 if T == 1 else 0
        ids = [torch.randint(0, 99092, (1, T), dtype=torch.int64, device=dev, generator=gi)
               for _ in range(8)]
        cache = torch.randint(0, 99092, (1, start + T + 8), dtype=torch.int64, device=dev,
                              generator=gi)

        def step(i, T=T, start=start):
            # up to replicate_max_tokens one launch reading the peers' shards in place;
            # above it the hasher, then the sliced gather-sum and its all-gather
            return hasher.lookup_sum(emb, ids[i % 8], start, cache)

        for i in range(args.warmup):
            step(i)
        torch.cuda.synchronize()
        dist.barrier()
        # up to replicate_max_tokens every rank sums all tokens and no collective runs: the
        # step is replayed from CUDA graphs; above it the step (with its NCCL all-gather) runs
        # as direct launches
        graphs = None
        if T <= emb.replicate_max_tokens:
            graphs = graphed(torch, [lambda c=c: step(c) for c in range(8)])
            run = lambda i: graphs[i % 8].replay()
        else:
            run = step
        with Clocks(local) as clk:
            ms = timed_steps(torch, run, args.steps, 0 if graphs is None else 3, flush, stream)
            dist.barrier()
            torch.cuda.synchronize()
        del graphs
        st = torch.tensor([statistics.median(ms)], device=dev)
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
        step_ms = float(st.item())
        byts = T * (24 * (d + 1) + 2 * d)
        res[f"engram_T{T}"] = {"ms": round(step_ms, 4), "tok_s": round(T / (step_ms / 1e3), 1),
                               "gbs_per_gpu": round(byts / world / (step_ms / 1e3) / 1e9, 1),
                               "clocks": clk.summary()}
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"metric": "engram hash + gather-sum tok/s (row-sharded table)",
                          "n_gpus": world, "parallelism": "rows%d" % world, "scaling": "strong",
                          "table_rows": rows, "rows_per_gpu": emb.part,
                          "peak_source": peak_src + " hbm_gbs", "hbm_peak": hbm_peak, **res}))


# ---------------------------------------------------------------- CPU baseline --

def cpu_baseline(seconds=15.0, sample_experts=None):
    """The numpy oracle (port of deepseek_v41_mlx moe/dequant) on the host cores for
    the same T=64 batch: router + shared expert in full, routed experts on a sample
    of the active experts, scaled to all of them."""
    import numpy as np
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import formats as F
    from oracle import moe as OM
    rng = np.random.default_rng(0)
    x = F.bf16_bits_to_f32(F.f32_to_bf16_bits(rng.standard_normal((T_HEAD, D)).astype(np.float32)))
    gw = F.bf16_bits_to_f32(F.f32_to_bf16_bits(
        (rng.standard_normal((E, D)) * D ** -0.5).astype(np.float32)))
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)

    def fp4(n, k):
        return (rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8),
                rng.integers(120, 129, size=(n, k // 32), dtype=np.uint8))

    def fp8(n, k):
        w = rng.integers(0, 256, size=(n, k), dtype=np.uint8)
        w[(w & 0x7F) == 0x7F] = 0
        return w, rng.integers(118, 128, size=(n // 32, k // 32), dtype=np.uint8)

    t0 = time.perf_counter()
    w, idx, _ = OM.gate(x, gw, bias, TOPK, acc=np.float32)
    t_router = time.perf_counter() - t0
    sh = {}
    for key, (n, k) in (("1", (I, D)), ("3", (I, D)), ("2", (D, I))):
        sh["sw" + key], sh["ss" + key] = fp8(n, k)
    t0 = time.perf_counter()
    OM.shared_expert_fp8(x, sh["sw1"], sh["ss1"], sh["sw3"], sh["ss3"], sh["sw2"], sh["ss2"],
                         10.0, True, np.float32)
    t_shared = time.perf_counter() - t0
    experts = np.unique(idx)
    done, t_exp = 0, 0.0
    for e in experts:
        w1, s1 = fp4(I, D)
        w3, s3 = fp4(I, D)
        w2, s2 = fp4(D, I)
        t_sel = np.nonzero((idx == e).any(-1))[0]
        t0 = time.perf_counter()
        OM.expert_fp4(x[t_sel], w1, s1, w3, s3, w2, s2, 10.0, True, np.float32)
        t_exp += time.perf_counter() - t0
        done += 1
        if sample_experts is not None and done >= sample_experts:
            break
        if sample_experts is None and t_exp + t_router + t_shared > seconds:
            break
    est = t_router + t_shared + t_exp * len(experts) / done
    cores = os.cpu_count()
    return {"value": round(T_HEAD / est, 4), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"T=64 batch: router + shared expert in full, {done} of {len(experts)} active "
                      f"routed experts timed and scaled linearly (numpy fp32, BLAS threads={cores})",
            "est_step_s": round(est, 3)}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    res = [cpu_baseline(sample_experts=args.ref_sample) for _ in range(args.warmup)]
    t0 = time.perf_counter()
    res = [cpu_baseline(sample_experts=args.ref_sample) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    est = statistics.mean(r["est_step_s"] for r in res)
    v = round(T_HEAD / est, 4)
    cpu = dict(res[-1])
    cpu["value"] = v
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(est * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 (numpy)", "impl": "reference",
        "data": "synthetic", "config": {"workload": "moe_decode_fp4 (BASELINE.json configs[1]) at T=64",
                                        "experts": E, "dim": D, "moe_inter_dim": I, "topk": TOPK},
        "cpu_baseline": cpu, "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0,
                                     "d2h_bytes_per_step": 0},
        "wall_s": round(wall, 1)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-sub", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--ref-sample", type=int, default=2, help="routed experts per reference step")
    ap.add_argument("--experts", type=int, default=384,
                    help="routed experts (384 = BASELINE; smaller only for ncu captures)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only the T=8192 a8 prefill measurement (one JSON line)")
    ap.add_argument("--prefill-tokens", type=int, default=8192)
    ap.add_argument("--affine-only", action="store_true",
                    help="only the M=4096 affine tensor-core measurement (one JSON line)")
    ap.add_argument("--engram-only", action="store_true",
                    help="only the engram d5 measurement (one JSON line)")
    ap.add_argument("--engram-vocab", type=int, default=4_000_000,
                    help="engram_vocab_size of d5 (4,000,000 = BASELINE; smaller only for ncu "
                         "captures)")
    args = ap.parse_args()
    global E, ROUTER_BYTES
    E = args.experts
    ROUTER_BYTES = E * D * 2
    if args.prefill_only and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_prefill_ep(args)
        return
    if args.prefill_only:
        import torch
        q = _package()
        dev = torch.device("cuda", 0)
        layer = make_moe(q, torch, dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        with Clocks(0) as clk:
            r = prefill_measurement(q, torch, dev, layer, flush, torch.cuda.current_stream(),
                                    _peaks(), args.steps, args.warmup, T=args.prefill_tokens)
        r["clocks"] = clk.summary()
        print(json.dumps(r))
        return
    if args.engram_only and int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_engram_ep(args)
        return
    if args.engram_only:
        import torch
        q = _package()
        dev = torch.device("cuda", 0)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        with Clocks(0) as clk:
            r = engram_measurement(q, torch, dev, flush, torch.cuda.current_stream(),
                                   args.steps, args.warmup, args.engram_vocab)
        r["clocks"] = clk.summary()
        print(json.dumps(r))
        return
    if args.affine_only:
        import torch
        q = _package()
        dev = torch.device("cuda", 0)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        with Clocks(0) as clk:
            r = affine_prefill_measurement(q, torch, dev, flush, torch.cuda.current_stream(),
                                           args.steps, args.warmup)
        r["clocks"] = clk.summary()
        print(json.dumps(r))
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
