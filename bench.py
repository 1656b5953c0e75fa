"""Benchmark of the quantized-weight hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline: a step is one MoE-layer forward at decode (router + fp4 routed experts + fp8
shared expert + combine) over one batch of T=64 tokens of synthetic bf16 activations,
with random-init weights of the release layout: 384 experts, dim 7168, moe_inter_dim
2048, top-6, ue8m0 scales in [120, 128].  ``value`` is
whole-job tokens/s with inputs resident in HBM; ``e2e`` is the same step through the
public API (``MoE.__call__``; ``EPMoE.forward`` at N > 1) with pinned host input/output
buffers copied inside the timed region.

Every other BASELINE config has its own entry under ``sub`` with the same three parts:
the metric with device-resident inputs plus the ``roofline`` of its dominant kernel, the
metric through the public API with host buffers (``e2e``), and the numpy port of the
reference's algorithm on the host cores (``cpu_baseline``):
  d1  fp8 dense linear [4096 x 7168], M = 1 / 32         (configs[0])  GB/s
  d2  the decode layer at T = 1 / 8 / 64                   (configs[1])  tok/s
  d3  the layer at prefill, T = 8192, Zipf(1.1) routing   (configs[2])  tok/s, TFLOP/s
  d4  MLX affine [14336 x 7168] 4 / 8 bit, M = 1/16/4096  (configs[3])  GB/s, TFLOP/s
  d5  engram hash + row gather-sum, T = 1 / 8192           (configs[4])  tok/s, GB/s
At N > 1 the headline is the expert-parallel decode layer, ``sub`` holds the
expert-parallel prefill (d3) and the row-sharded engram table (d5), and each of the three
carries an ``ep_check``: the sharded result against rank 0's single-GPU result on the same
inputs (a mismatch beyond the GEMV tolerance fails the run).

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and
torch.cuda.synchronize(); each step is timed with CUDA events on the launching stream; L2
is flushed (256 MiB write) between steps outside the events and input batches rotate.
Kernel durations for the roofline come from CUDA events the library records around each
launch on its stream.  Multi-GPU: one process per GPU (torchrun), max over ranks.

--impl reference times the reference's CPU algorithm for the headline step (the numpy
oracle restating deepseek_v41_mlx/moe.py + dequant.py; the MLX original cannot be
installed offline) on the host cores: whole T=64 steps, as many as fit its time budget.
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
D1_N, D1_K = 4096, 7168                                  # configs[0]
D4_N, D4_K = 14336, 7168                                 # configs[3]
ENGRAM_DIM, ENGRAM_ROWS_PER_TOKEN = 1024, 24             # configs[4]
PREFILL_T = 8192                                         # configs[2]


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


def _traffic(key, units=1.0):
    """DRAM bytes (read + write) of one launch from an ncu capture summarised in
    profiles/traffic.json, scaled by the units the launch processes; None if not captured."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    ent = json.load(open(p)).get(key)
    if not ent:
        return None
    if "dram_bytes_per_unit" in ent:
        return int(ent["dram_bytes_per_unit"] * units)
    if "dram_bytes_per_active_expert" in ent:
        return int(ent["dram_bytes_per_active_expert"] * units)
    return int(ent["dram_bytes_per_launch"])


def _roofline(bound, kernel, work, launch_ms, peak, peak_src, traffic=None):
    """Roofline of one kernel: algorithmic bytes (bound "hbm", GB/s) or FLOPs (bound
    "tensor", TFLOP/s) per launch over its average launch time."""
    if not launch_ms:
        return None
    if bound == "hbm":
        ach = work / (launch_ms / 1e3) / 1e9
        unit, key = "GB/s", "algorithmic_bytes"
    else:
        ach = work / (launch_ms / 1e3) / 1e12
        unit, key = "TFLOP/s", "algorithmic_flops"
    return {"bound": bound, "kernel": kernel, "achieved": round(ach, 1), "peak": peak,
            "unit": unit, "frac": round(ach / peak, 4), "traffic": traffic, key: int(work),
            "avg_launch_ms": round(launch_ms, 5), "peak_source": peak_src}


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
    n_exp = gate_w.shape[0]
    perm = torch.randperm(n_exp, device=dev, generator=g)
    logp = torch.empty(n_exp, device=dev)
    logp[perm] = -s * torch.log(torch.arange(1, n_exp + 1, device=dev, dtype=torch.float32))
    u = torch.rand(T, n_exp, device=dev, generator=g).clamp_(1e-30, 1.0)
    idx = (logp[None, :] - torch.log(-torch.log(u))).topk(TOPK, dim=-1).indices
    scores = torch.sqrt(torch.nn.functional.softplus(x.float() @ gate_w.float().T))
    w = scores.gather(1, idx)
    w = w / (w.sum(-1, keepdim=True) + 1e-20) * 1.5
    return w.contiguous(), idx.to(torch.int32).contiguous()


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


def kernel_ms(q, torch, fn, names, K, flush, stream):
    """Average device time per launch of each named kernel over K direct calls of ``fn``
    (CUDA events the library records on the launching stream around each launch), with L2
    flushed before every call.  -> {name: (launches per call, ms per launch)}."""
    q._lib.prof_enable(True)
    q._lib.prof_select(list(names))
    try:
        for i in range(K):
            flush.zero_()
            fn(i)
        torch.cuda.synchronize()
        rep = q._lib.prof_report()
    finally:
        q._lib.prof_select(None)
        q._lib.prof_enable(False)
    return {k: (v[0] / K, v[1] / v[0]) for k, v in rep.items() if v[0]}


def capture(torch, fn):
    """fn's launches as a CUDA graph; Python's cycle collector runs first and is off during the
    capture, so that no finalizer destroys a CUDA graph or event inside it."""
    import gc
    g = torch.cuda.CUDAGraph()
    gc_on = gc.isenabled()
    gc.collect()
    gc.disable()
    try:
        with torch.cuda.graph(g):
            fn()
    finally:
        if gc_on:
            gc.enable()
    return g


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
        out.append(capture(torch, f))
    return out


def e2e_measure(torch, fn, host_in, dev_in, out_host, K, W, flush, stream):
    """The call through the public API with its inputs copied from pinned host buffers and
    its result read back to a pinned host buffer, both inside each timed step.
    ``host_in``/``dev_in``: lists of (pinned host, device) tensors (rotated per step for
    lists of lists); ``fn(i)`` returns the device result.  -> (mean ms, h2d B, d2h B)."""
    def step(i):
        src = host_in[i % len(host_in)]
        for h, d in zip(src, dev_in):
            d.copy_(h, non_blocking=True)
        y = fn(i)
        out_host.copy_(y, non_blocking=True)
    ms = timed_steps(torch, step, K, W, flush, stream)
    h2d = sum(h.numel() * h.element_size() for h in host_in[0])
    return statistics.mean(ms), h2d, out_host.numel() * out_host.element_size()


# ---------------------------------------------------------------- d1: fp8 dense GEMV --

def d1_measure(q, torch, dev, flush, stream, K, W, peaks, ms_list=(1, 32)):
    hbm, _, src = peaks
    N, Kd = D1_N, D1_K
    g = torch.Generator(device=dev).manual_seed(11)
    copies = 10                                  # 294 MB of weights rotated (> 2x L2)
    ws = [torch.randint(0, 256, (N, Kd), dtype=torch.uint8, device=dev, generator=g)
          for _ in range(copies)]
    ss = [torch.randint(118, 128, (N // 32, Kd // 32), dtype=torch.uint8, device=dev, generator=g)
          for _ in range(copies)]
    for w in ws:
        w[(w & 0x7F) == 0x7F] = 0
    out = {}
    for M in ms_list:
        x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
        byts = N * Kd + (N // 32) * (Kd // 32) + M * Kd * 2 + M * N * 2
        gr = graphed(torch, [lambda c=c: q.linear.linear_fp8(x, ws[c], ss[c]) for c in range(copies)])
        st = statistics.mean(timed_steps(torch, lambda i: gr[i % copies].replay(), K * 4, W, flush,
                                         stream))
        # one activation row: the single-launch CUDA-core kernel; more: the tensor-core engine
        kname = "gemv_fp8_m1" if M == 1 else "qgemv_dense"
        klabel = ("gemv_fp8_m1 (k_gemv_fp8_m1)" if M == 1
                  else "qgemv_dense (k_qgemv<FP8B,1,NT>)")
        kt = kernel_ms(q, torch, lambda i: q.linear.linear_fp8(x, ws[i % copies], ss[i % copies]),
                       [kname, "qx_prep"], K * 2, flush, stream)
        # the GEMV over the 10 weight copies back to back in one graph (a decode step runs
        # many such products in a row): time per GEMV
        chain = graphed(torch, [lambda: [q.linear.linear_fp8(x, ws[c], ss[c])
                                         for c in range(copies)]])[0]
        stc = statistics.mean(timed_steps(torch, lambda i: chain.replay(), K, W, flush,
                                          stream)) / copies
        xh = [[x.cpu().pin_memory()]]
        xd = torch.empty_like(x)
        yh = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
        e_ms, bi, bo = e2e_measure(torch, lambda i: q.linear.linear_fp8(xd, ws[i % copies],
                                                                         ss[i % copies]),
                                   xh, [xd], yh, K * 2, W, flush, stream)
        gk = kt.get(kname, (0, None))[1]
        out[f"gemv_fp8_block_M{M}"] = {
            "config": f"BASELINE.json configs[0]: fp8 e4m3 [{N} x {Kd}], ue8m0 32x32, M={M}, "
                      f"bf16 out; {copies} weight copies rotated",
            "metric": "dequant-GEMV HBM GB/s", "unit": "GB/s",
            "value": round(byts / st / 1e6, 1), "ms": round(st, 5),
            "frac_hbm": round(byts / st / 1e6 / hbm, 4),
            "chained_ms": round(stc, 5), "chained_gbs": round(byts / stc / 1e6, 1),
            "chained_frac_hbm": round(byts / stc / 1e6 / hbm, 4),
            "kernel_ms": {k: round(v[1], 5) for k, v in kt.items()},
            "roofline": _roofline("hbm", klabel, byts, gk, hbm,
                                  src + " hbm_gbs (copy)", _traffic(f"{kname}_fp8_M{M}")),
            "e2e": {"value": round(byts / e_ms / 1e6, 1), "unit": "GB/s", "ms": round(e_ms, 5),
                    "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                    "api": "linear.linear_fp8"},
        }
        del gr, chain
    del ws, ss
    return out


# ---------------------------------------------------------------- d2: decode at T=1/8/64 --

def d2_measure(q, torch, dev, layer, flush, stream, K, W, peaks):
    hbm = peaks[0]
    out = {}
    g = torch.Generator(device=dev).manual_seed(99)
    layer.cuda_graph = True
    for T in (1, 8, 64):
        xs = [torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(8)]
        ms = timed_steps(torch, lambda i: layer(xs[i % 8]), K, W, flush, stream)
        act = statistics.mean(len(torch.unique(layer(x, with_routing=True)[2])) for x in xs[:4])
        st = statistics.mean(ms)
        byts = act * BYTES_PER_EXPERT + ROUTER_BYTES + SHARED_BYTES
        out[f"moe_decode_T{T}_graph"] = {"tok_s": round(T / (st / 1e3), 1), "ms": round(st, 4),
                                         "active_experts": round(act, 1),
                                         "layer_gbs": round(byts / (st / 1e3) / 1e9, 1),
                                         "frac_hbm": round(byts / (st / 1e3) / 1e9 / hbm, 4)}
    layer.cuda_graph = False
    return out


# ---------------------------------------------------------------- d3: prefill --

PF_ROUTED = ("pf_gate_up_fp4", "pf_gate_up_fp4_narrow", "pf_down_fp4", "pf_down_fp4_narrow")


def prefill_measurement(q, torch, dev, layer, flush, stream, peaks, K, W, T=PREFILL_T,
                        e2e=True):
    """d3: the layer at prefill in a8 numerics (upstream linear()), T=8192, Zipf routing.
    The routed grouped GEMMs run on four kernels (gate/up and down, each on wide tiles for
    heavily routed experts and narrow tiles for light ones); all four count."""
    hbm_peak, bf16_peak, peak_src = peaks
    g = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = zipf_routing(torch, dev, x, layer.gate.weight, T)
    counts = torch.bincount(idx.reshape(-1).long(), minlength=E)
    fn = lambda i: layer.prefill_a8(x, weights=w, indices=idx)
    st = statistics.median(timed_steps(torch, fn, K, W, flush, stream))
    kt = kernel_ms(q, torch, fn, [], max(3, K // 2), flush, stream)    # every kernel
    f_routed = 2.0 * T * TOPK * 3 * I * D
    f_shared = 2.0 * 3 * T * I * D
    fp8_peak = 2.0 * bf16_peak          # f8f6f4 rate = twice the bf16 rate
    kern = {k: round(v[1] * v[0], 4) for k, v in kt.items()}           # ms per layer call
    routed_ms = sum(kern.get(k, 0.0) for k in PF_ROUTED)
    active = int((counts > 0).sum())
    wbytes = active * BYTES_PER_EXPERT
    # the routed GEMMs stream every active expert's weights (HBM) and do 4.33 TFLOP
    # (tensor): their roofline time is the larger of the two
    floor_ms = max(f_routed / (fp8_peak * 1e12), wbytes / (hbm_peak * 1e9)) * 1e3
    r = {
        "config": "BASELINE.json configs[2]: T=8192 bf16 N(0,1), Zipf(1.1) top-6 routing, fp4 "
                  "experts 384 x [2048 x 7168], a8 (upstream act_quant + block-scaled MMA)",
        "metric": "MoE-layer prefill tok/s", "unit": "tok/s",
        "value": round(T / (st / 1e3), 1), "tok_s": round(T / (st / 1e3), 1), "ms": round(st, 4),
        "tokens": T, "tflops_layer": round((f_routed + f_shared) / (st / 1e3) / 1e12, 1),
        "routed_gemm_ms": round(routed_ms, 4),
        "routed_gemm_tflops": round(f_routed / (routed_ms / 1e3) / 1e12, 1) if routed_ms else None,
        "routed_gemm_frac_fp8_peak": round(f_routed / (routed_ms / 1e3) / 1e12 / fp8_peak, 4)
        if routed_ms else None,
        "routed_roofline_ms": round(floor_ms, 4),
        "routed_frac_of_roofline": round(floor_ms / routed_ms, 4) if routed_ms else None,
        "routed_weight_gbs": round(wbytes / (routed_ms / 1e3) / 1e9, 1) if routed_ms else None,
        "fp8_peak_tflops": fp8_peak, "peak_source": peak_src + " 2x bf16_tflops (f8f6f4 rate)",
        "kernel_ms": kern, "experts_active": active, "pairs_max_expert": int(counts.max()),
        "pairs_min_expert": int(counts.min()),
        "routing": "Zipf(1.1) Gumbel-top-6 over a seeded expert permutation; router-score weights",
        "roofline": _roofline("tensor", "routed grouped GEMMs (k_bsgemm: 4 launches, wide + "
                              "narrow tiles)", f_routed, routed_ms, fp8_peak,
                              peak_src + " 2x bf16_tflops (f8f6f4 rate)",
                              _traffic("pf_routed_gemms", active)),
    }
    if e2e:
        xh = [[x.cpu().pin_memory(), w.cpu().pin_memory(), idx.cpu().pin_memory()]]
        xd, wd, idd = torch.empty_like(x), torch.empty_like(w), torch.empty_like(idx)
        yh = torch.empty((T, D), dtype=torch.bfloat16).pin_memory()
        e_ms, bi, bo = e2e_measure(torch, lambda i: layer.prefill_a8(xd, weights=wd, indices=idd),
                                   xh, [xd, wd, idd], yh, max(3, K // 2), W, flush, stream)
        r["e2e"] = {"value": round(T / (e_ms / 1e3), 1), "unit": "tok/s", "ms": round(e_ms, 4),
                    "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                    "api": "moe.MoE.prefill_a8(x, weights, indices)"}
    return r


A16_ROUTED = ("a16_gate_up_fp4", "a16_down_fp4")


def prefill_a16_measurement(q, torch, dev, layer, flush, stream, peaks, K, W, T=PREFILL_T,
                            e2e=True):
    """d3 in the port's numerics (MoE.prefill_a16): bf16 activations x exactly decoded
    weights on kind::f16 tensor cores, the routed down projection on the fp32 SwiGLU output as
    bf16 hi + lo (two MMAs a K step), so the routed GEMMs execute 4/3 of the layer's 4.33
    TFLOP; measured against the bf16 peak with the model's FLOPs."""
    hbm_peak, bf16_peak, peak_src = peaks
    g = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = zipf_routing(torch, dev, x, layer.gate.weight, T)
    counts = torch.bincount(idx.reshape(-1).long(), minlength=E)
    fn = lambda i: layer.prefill_a16(x, weights=w, indices=idx)
    st = statistics.median(timed_steps(torch, fn, K, W, flush, stream))
    kt = kernel_ms(q, torch, fn, [], max(3, K // 2), flush, stream)
    f_routed = 2.0 * T * TOPK * 3 * I * D
    f_shared = 2.0 * 3 * T * I * D
    kern = {k: round(v[1] * v[0], 4) for k, v in kt.items()}
    routed_ms = sum(kern.get(k, 0.0) for k in A16_ROUTED)
    active = int((counts > 0).sum())
    wbytes = active * BYTES_PER_EXPERT
    floor_ms = max(f_routed / (bf16_peak * 1e12), wbytes / (hbm_peak * 1e9)) * 1e3
    r = {
        "config": "BASELINE.json configs[2] in the port's numerics (deepseek_v41_mlx/moe.py): T=8192 "
                  "bf16 N(0,1), Zipf(1.1) top-6 routing, fp4 experts 384 x [2048 x 7168], bf16 "
                  "activations (no act_quant), gate/up rounded to bf16",
        "metric": "MoE-layer prefill tok/s (port numerics)", "unit": "tok/s",
        "value": round(T / (st / 1e3), 1), "ms": round(st, 4), "tokens": T,
        "tflops_layer": round((f_routed + f_shared) / (st / 1e3) / 1e12, 1),
        "routed_gemm_ms": round(routed_ms, 4),
        "routed_gemm_tflops": round(f_routed / (routed_ms / 1e3) / 1e12, 1) if routed_ms else None,
        "routed_executed_tflops": round(f_routed * 4 / 3 / (routed_ms / 1e3) / 1e12, 1)
        if routed_ms else None,
        "routed_roofline_ms": round(floor_ms, 4),
        "routed_frac_of_roofline": round(floor_ms / routed_ms, 4) if routed_ms else None,
        "kernel_ms": kern, "experts_active": active,
        "roofline": _roofline("tensor", "routed a16 GEMMs (k_a16gemm: gate/up + down, wide and "
                              "narrow tile lists)", f_routed, routed_ms, bf16_peak,
                              peak_src + " bf16_tflops (cuBLAS burst)"),
    }
    if e2e:
        xh = [[x.cpu().pin_memory(), w.cpu().pin_memory(), idx.cpu().pin_memory()]]
        xd, wd, idd = torch.empty_like(x), torch.empty_like(w), torch.empty_like(idx)
        yh = torch.empty((T, D), dtype=torch.bfloat16).pin_memory()
        e_ms, bi, bo = e2e_measure(torch, lambda i: layer.prefill_a16(xd, weights=wd, indices=idd),
                                   xh, [xd, wd, idd], yh, max(3, K // 2), W, flush, stream)
        r["e2e"] = {"value": round(T / (e_ms / 1e3), 1), "unit": "tok/s", "ms": round(e_ms, 4),
                    "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
                    "api": "moe.MoE.prefill_a16(x, weights, indices)"}
    return r


# ---------------------------------------------------------------- d4: MLX affine --

def d4_measure(q, torch, dev, flush, stream, K, W, peaks):
    hbm, bf16_peak, src = peaks
    N, Kd = D4_N, D4_K
    g = torch.Generator(device=dev).manual_seed(77)
    out = {}
    for bits in (4, 8):
        copies = 4 if bits == 4 else 3
        wq = [torch.randint(-2 ** 31, 2 ** 31 - 1, (N, Kd * bits // 32), dtype=torch.int32,
                            device=dev, generator=g) for _ in range(copies)]
        sc = [(torch.rand(N, Kd // 64, device=dev, generator=g) * 0.019 + 0.001).to(torch.bfloat16)
              for _ in range(copies)]
        bi = [(torch.randn(N, Kd // 64, device=dev, generator=g) * 0.05).to(torch.bfloat16)
              for _ in range(copies)]
        call = lambda x, c: q.linear.linear_affine(x, wq[c], sc[c], bi[c], bits)
        for M in (1, 16, 4096):
            x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
            if M <= 16:
                byts = N * Kd * bits // 8 + 2 * N * (Kd // 64) * 2 + M * Kd * 2 + M * N * 2
                gr = graphed(torch, [lambda c=c: call(x, c) for c in range(copies)])
                st = statistics.mean(timed_steps(torch, lambda i: gr[i % copies].replay(), K * 4,
                                                 W, flush, stream))
                del gr
                kname = f"gemv_affine{bits}_m1" if M == 1 else "qgemv_dense"
                bound, work, pk = "hbm", byts, hbm
                metric, unit = "dequant-GEMV HBM GB/s", "GB/s"
                val = byts / st / 1e6
            else:
                flops = 2.0 * M * N * Kd
                st = statistics.median(timed_steps(torch, lambda i: call(x, i % copies), K, W,
                                                   flush, stream))
                kname, bound, work, pk = "qmm_affine", "tensor", flops, bf16_peak
                metric, unit = "affine quantized matmul TFLOP/s", "TFLOP/s"
                val = flops / (st / 1e3) / 1e12
            kt = kernel_ms(q, torch, lambda i: call(x, i % copies), [kname], max(3, K),
                           flush, stream)
            xh = [[x.cpu().pin_memory()]]
            xd = torch.empty_like(x)
            yh = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
            e_ms, hb, db = e2e_measure(torch, lambda i: call(xd, i % copies), xh, [xd], yh,
                                       max(3, K), W, flush, stream)
            e_val = work / e_ms / 1e6 if bound == "hbm" else work / (e_ms / 1e3) / 1e12
            kms = kt.get(kname, (0, None))[1]
            out[f"affine{bits}_M{M}"] = {
                "config": f"BASELINE.json configs[3]: MLX affine {bits}-bit g64 [{N} x {Kd}], "
                          f"bf16 scale/bias, M={M}" + (f"; {copies} weight copies rotated"
                                                      if M <= 16 else ""),
                "metric": metric, "unit": unit, "value": round(val, 1), "ms": round(st, 5),
                "frac_peak": round(val / pk, 4),
                "kernel_ms": {k: round(v[1], 5) for k, v in kt.items()},
                "roofline": _roofline(bound, kname, work, kms, pk,
                                      src + (" hbm_gbs (copy)" if bound == "hbm"
                                             else " bf16_tflops (cuBLAS burst)"),
                                      _traffic(f"{kname}_affine{bits}_M{M}")),
                "e2e": {"value": round(e_val, 1), "unit": unit, "ms": round(e_ms, 5),
                        "h2d_bytes_per_step": hb, "d2h_bytes_per_step": db,
                        "api": "linear.linear_affine"},
            }
        del wq, sc, bi
    # converter (next row 3): mx.quantize of a bf16 [14336, 7168] weight, groups of 64; two
    # weight copies (> L2) rotated; bytes = bf16 in + codes + bf16 scales and biases out
    ws_bf = [torch.randn(N, Kd, device=dev, generator=g).to(torch.bfloat16) for _ in range(2)]
    for bits in (4, 8):
        gr = graphed(torch, [lambda c=c: q.dequant.quantize_affine(ws_bf[c], 64, bits)
                             for c in range(2)])
        st = statistics.mean(timed_steps(torch, lambda i: gr[i % 2].replay(), K * 2, W, flush,
                                         stream))
        byts = N * Kd * 2 + N * Kd * bits // 8 + 2 * N * (Kd // 64) * 2
        out[f"quantize_affine{bits}_14336x7168"] = {
            "ms": round(st, 4), "gbs": round(byts / st / 1e6, 1),
            "frac_hbm": round(byts / st / 1e6 / hbm, 4)}
        del gr
    del ws_bf
    return out


# ---------------------------------------------------------------- d5: engram --

def _engram_args(vocab):
    import types
    return types.SimpleNamespace(engram_layer_ids=(1,), engram_max_ngram_size=4,
                                 engram_vocab_size=vocab, engram_n_heads=8, engram_pad_id=2,
                                 engram_compressed_vocab_size=99092)


def engram_measurement(q, torch, dev, flush, stream, K, W, vocab=4_000_000, peaks=None,
                       tokens=(1, PREFILL_T)):
    """d5: engram table fp8 e4m3 [96,000,xxx x 1024] (one ue8m0 per row, [115, 127]) built on
    the device, 24 rows per token (2/3/4-gram x 8 heads, one layer, primes from 4,000,000)
    hashed from uniform compressed ids in [0, 99092); a step = hash + gather + dequant + fp32
    sum -> bf16 [T, 1024] through EngramHasher.lookup_sum (one launch up to its
    fused_max_positions, the hasher then the gather-sum above); ``ms_two_step`` always times
    the latter.  Bytes per token: 24 x (1024 + 1) read + 2048 written.  A smaller ``vocab``
    (engram_vocab_size) gives a table of about 24 x vocab rows, for ncu captures."""
    import numpy as np
    hbm_peak, _, peak_src = peaks or _peaks()
    args = _engram_args(vocab)
    primes, _ = q.engram.build_layout(args)
    rows, d = int(primes.sum()), ENGRAM_DIM
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
    for T in tokens:
        start = 100 if T == 1 else 0
        ids = [torch.randint(0, 99092, (1, T), dtype=torch.int64, device=dev, generator=g)
               for _ in range(8)]
        cache = torch.randint(0, 99092, (1, start + T + 8), dtype=torch.int64, device=dev,
                              generator=g)

        def step(i, start=start):
            # hash + gather-sum (one launch up to EngramHasher.fused_max_positions positions)
            return hasher.lookup_sum(emb, ids[i % 8], start, cache)

        def step2(i, T=T, start=start):
            idx = hasher(ids[i % 8], start, cache)
            return emb.gather_sum(idx.reshape(T, -1))

        # the step replayed from CUDA graphs (one per input batch): device time, no host gaps
        gr = graphed(torch, [lambda c=c: step(c) for c in range(8)])
        ms = statistics.median(timed_steps(torch, lambda i: gr[i % 8].replay(), K, W, flush,
                                           stream))
        del gr
        ms_host = statistics.median(timed_steps(torch, step, K, W, flush, stream))
        gr2 = graphed(torch, [lambda c=c: step2(c) for c in range(8)])
        ms2 = statistics.median(timed_steps(torch, lambda i: gr2[i % 8].replay(), K, W, flush,
                                            stream))
        del gr2
        fused = T <= hasher.fused_max_positions
        kname = "engram_lookup_sum" if fused else "engram_gather_sum"
        kt = kernel_ms(q, torch, step, ["engram_lookup_sum", "engram_gather_sum", "engram_hash"],
                       max(3, K), flush, stream)
        byts = T * (ENGRAM_ROWS_PER_TOKEN * (d + 1) + 2 * d)
        ih = [[ids[c].cpu().pin_memory()] for c in range(8)]
        idd = torch.empty_like(ids[0])
        oh = torch.empty((1, T, d), dtype=torch.bfloat16).pin_memory()
        e_ms, hb, db = e2e_measure(torch, lambda i: hasher.lookup_sum(emb, idd, start, cache),
                                   ih, [idd], oh, max(3, K), W, flush, stream)
        out[f"engram_T{T}"] = {
            "config": f"BASELINE.json configs[4]: fp8 table [{rows} x {d}] + ue8m0 per row "
                      f"(packed, {rb} B rows, {rows * rb / 1e9:.1f} GB on one GPU), 24 rows a "
                      f"token, T={T}",
            "metric": "engram hash + gather-sum tok/s", "unit": "tok/s",
            "value": round(T / (ms / 1e3), 1), "ms": round(ms, 4),
            "ms_eager": round(ms_host, 4), "ms_two_step": round(ms2, 4),
            "tok_s": round(T / (ms / 1e3), 1), "gbs": round(byts / (ms / 1e3) / 1e9, 1),
            "frac_hbm": round(byts / (ms / 1e3) / 1e9 / hbm_peak, 4),
            "kernel_ms": {k: round(v[1], 5) for k, v in kt.items()},
            "roofline": _roofline("hbm", kname, byts, kt.get(kname, (0, None))[1], hbm_peak,
                                  peak_src + " hbm_gbs (copy)", _traffic(kname + "_rows", T)),
            "table_rows": rows, "table_gb": round(rows * rb / 1e9, 1),
            "table_layout": "packed rows (codes + scale, %d B)" % rb,
            "e2e": {"value": round(T / (e_ms / 1e3), 1), "unit": "tok/s", "ms": round(e_ms, 4),
                    "h2d_bytes_per_step": hb, "d2h_bytes_per_step": db,
                    "api": "engram.EngramHasher.lookup_sum"},
        }
    del table, emb
    torch.cuda.empty_cache()
    return out


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
    peaks = _peaks()
    hbm_peak, bf16_peak, peak_src = peaks
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

    ep_check = None
    if world > 1:
        ep_check = ep_check_decode(q, torch, dist, dev, layer, rank, world)

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
            steps.append(capture(torch, lambda i=i: fwd(xs[i % len(xs)])))
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
    # per-kernel breakdown (every kernel bracketed by events): a separate, untimed pass; at
    # N > 1 a barrier before each step, so that the waits on peers' flags measure the
    # exchange and not the ranks' skew in starting the step
    q._lib.prof_enable(True)
    if world > 1:
        def kstep(i):
            torch.cuda.synchronize()
            dist.barrier()
            fwd(xs[i % len(xs)])
    else:
        kstep = lambda i: fwd(xs[i % len(xs)])
    timed_steps(torch, kstep, max(3, K // 4), 0, flush, stream)
    kprof = q._lib.prof_report()
    q._lib.prof_enable(False)
    step_ms = sum(ms) / len(ms)
    if world > 1:
        t = torch.tensor([step_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms = float(t.item())
    value = T_HEAD * world / (step_ms / 1e3)

    # active experts per step (for the algorithmic byte count), outside timing: at N > 1
    # each rank streams its own experts that the step's pairs reach (counted over the
    # NCCL form of the exchange, which every rank runs the same number of times)
    active, local_active = [], None
    if world > 1:
        layer.track = True
        for x in xs[:4]:
            layer.forward(x)
        layer.track = False
        la = torch.tensor([layer.local_active_mean], device=dev)
        every = [torch.zeros_like(la) for _ in range(world)]
        dist.all_gather(every, la)
        local_active = [float(v.item()) for v in every]
        for x in xs[:4]:
            _, _, idx = layer.full_routing(x)
            ids = [torch.empty_like(idx) for _ in range(world)]
            dist.all_gather(ids, idx)
            active.append(len(torch.unique(torch.cat(ids))))
    else:
        for x in xs[:4]:
            _, _, idx = fwd(x, with_routing=True)
            active.append(len(torch.unique(idx)))
    n_act = statistics.mean(active)

    gu = prof.get("moe_expert_gate_up_fp4")
    roof = None
    if gu:
        gu_ms = gu[1] / gu[0]
        n_act_local = n_act if world == 1 else layer.local_active_mean
        gu_bytes = n_act_local * GU_BYTES_PER_EXPERT
        roof = _roofline("hbm", "moe_expert_gate_up_fp4", gu_bytes, gu_ms, hbm_peak,
                         peak_src + " hbm_gbs (copy)",
                         _traffic("moe_expert_gate_up_fp4", n_act_local))
    if world == 1:
        layer_bytes = n_act * BYTES_PER_EXPERT + ROUTER_BYTES + SHARED_BYTES
    else:           # every rank streams its local active experts + router + shared expert
        layer_bytes = sum(local_active) * BYTES_PER_EXPERT + world * (ROUTER_BYTES + SHARED_BYTES)
    layer_gbs = layer_bytes / (step_ms / 1e3) / 1e9

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
        Ks = max(3, K // 2)
        sub.update(d2_measure(q, torch, dev, layer, flush, stream, Ks, W, peaks))
        sub.update(d1_measure(q, torch, dev, flush, stream, Ks, W, peaks))
        sub.update(d4_measure(q, torch, dev, flush, stream, Ks, W, peaks))
        sub["moe_prefill_T8192_a8"] = prefill_measurement(
            q, torch, dev, layer, flush, stream, peaks, max(3, K // 4), W)
        sub["moe_prefill_T8192_a16"] = prefill_a16_measurement(
            q, torch, dev, layer, flush, stream, peaks, max(3, K // 4), W)
        layer = fwd = e2e_step = None          # the 99.8 GB engram table comes next
        torch.cuda.empty_cache()
        sub.update(engram_measurement(q, torch, dev, flush, stream, Ks, W, peaks=peaks))
    elif world > 1 and not args.no_sub:
        layer.close()                          # unmap the peers' exchange buffers (collective)
        layer = fwd = e2e_step = None
        torch.cuda.empty_cache()
        sub["moe_prefill_T8192_a8_ep"] = prefill_ep_measure(q, torch, dist, dev, rank, world,
                                                            args.steps, args.warmup, flush,
                                                            stream, peaks)
        sub.update(engram_ep_measure(q, torch, dist, dev, rank, world, args.steps, args.warmup,
                                     flush, stream, peaks))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_moe_baseline()
        if sub:
            cpu_sub_baselines(sub, args.cpu_seconds)

    checks_ok = True
    if world > 1:
        for c in [ep_check] + [v.get("ep_check") for v in sub.values() if isinstance(v, dict)]:
            if c is not None and not c.get("ok", True):
                checks_ok = False
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        if not checks_ok:
            sys.exit(1)
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "fp4-e2m1 weights x bf16 act (f16 mma, f32 acc)",
        "data": "synthetic (random-init weights of the release layout, N(0,1) bf16 activations)",
        "config": {"workload": "moe_decode_fp4 (BASELINE.json configs[1]) at T=64",
                   "experts": E, "dim": D, "moe_inter_dim": I, "topk": TOPK,
                   "tokens_per_gpu": T_HEAD, "global_batch": T_HEAD * world,
                   "parallelism": "ep%d" % world if world > 1 else "single",
                   "l2": "flushed (256 MiB write) between timed steps; inputs rotate over 8 batches",
                   "active_experts_mean": round(n_act, 1),
                   "active_experts_per_gpu": [round(v, 1) for v in local_active]
                   if local_active else None,
                   "layer_bytes_per_step": int(layer_bytes)},
        "roofline": roof,
        "layer_hbm_gbs": round(layer_gbs, 1),
        "layer_frac_hbm": round(layer_gbs / hbm_peak / world, 4),
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
        "kernel_ms": {k: round(v[1] / v[0], 5) for k, v in kprof.items()},
        "clocks": clk.summary(), "sub": sub,
    }
    if ep_check is not None:
        line["ep_check"] = ep_check
    print(json.dumps(line))
    if not checks_ok:
        sys.exit(1)


# ---------------------------------------------------------------- multi-GPU checks --

def _rel(a, b):
    import torch
    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / max(float(torch.linalg.vector_norm(b)), 1e-30))


def _verdict(torch, dist, dev, rank, res, tol):
    """rank 0's comparison -> every rank: {"bitwise", "max_rel", "ok"}."""
    t = torch.tensor(res if rank == 0 else [0.0, 0.0], dtype=torch.float64, device=dev)
    dist.broadcast(t, 0)
    bitwise, rel = bool(t[0].item()), float(t[1].item())
    return {"bitwise": bitwise, "max_rel": rel, "tol": tol, "ok": bitwise or rel < tol}


def ep_check_decode(q, torch, dist, dev, layer, rank, world):
    """One decode batch through the expert-parallel layer on every rank, against rank 0's
    single-GPU layer over all experts on the gathered tokens.  Both run the exact numerics
    (fp32 intermediates, fp32 output): a K split that depends on the batch (the shared
    expert's, at 64 tokens a rank against 64 x world on one GPU) then changes only the
    fp32 summation order, where the port's bf16 rounding of intermediates could turn such an
    order difference into a whole bf16 step."""
    from importlib import import_module
    ep = import_module("deepseek_v41_mlx_b200.ep")
    g = torch.Generator(device=dev).manual_seed(777 + rank)
    x = torch.randn(T_HEAD, D, device=dev, generator=g).to(torch.bfloat16)
    mode = layer.local.round_bf16
    layer.local.round_bf16 = False
    y = layer.forward(x.float())                       # fp32 out, peer-memory exchange
    layer.local.round_bf16 = mode
    xs = [torch.empty_like(x) for _ in range(world)]
    ys = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(xs, x)
    dist.all_gather(ys, y)
    res = None
    if rank == 0:
        full = ep.EPMoE.random_init_full(q, torch, dev, world, E, D, I, TOPK)
        full.round_bf16 = False
        yref = full(torch.cat(xs).float())
        yep = torch.cat(ys)
        res = [float(torch.equal(yref, yep)), _rel(yep, yref)]
        del full, yref
        torch.cuda.empty_cache()
    out = _verdict(torch, dist, dev, rank, res, 1e-5)
    out["tokens"] = T_HEAD * world
    return out


def prefill_ep_measure(q, torch, dist, dev, rank, world, K, W, flush, stream, peaks, T=PREFILL_T,
                       T_check=2048):
    """d3 over NCCL: each rank prefills its own T tokens (weak scaling) with E / ws experts;
    the step is timed with CUDA events per rank, max over ranks.  ep_check: T_check tokens
    per rank against rank 0's single-GPU layer on the gathered tokens and routing."""
    from importlib import import_module
    ep = import_module("deepseek_v41_mlx_b200.ep")
    hbm_peak, bf16_peak, peak_src = peaks
    layer = ep.EPMoE.random_init(q, torch, dev, rank, world, E, D, I, TOPK)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = zipf_routing(torch, dev, x, layer.gate_w, T, seed=7 + rank)
    # ---- check
    xc, wc, ic = x[:T_check].contiguous(), w[:T_check].contiguous(), idx[:T_check].contiguous()
    yc = layer.forward_prefill(xc, weights=wc, indices=ic, out_dtype=torch.float32)
    gx = [torch.empty_like(xc) for _ in range(world)]
    gw = [torch.empty_like(wc) for _ in range(world)]
    gi = [torch.empty_like(ic) for _ in range(world)]
    gy = [torch.empty_like(yc) for _ in range(world)]
    for a, b in ((gx, xc), (gw, wc), (gi, ic), (gy, yc)):
        dist.all_gather(a, b)
    res = None
    if rank == 0:
        full = ep.EPMoE.random_init_full(q, torch, dev, world, E, D, I, TOPK)
        yref = full.prefill_a8(torch.cat(gx), weights=torch.cat(gw), indices=torch.cat(gi),
                               out_dtype=torch.float32)
        yep = torch.cat(gy)
        res = [float(torch.equal(yref, yep)), _rel(yep, yref)]
        del full, yref
        torch.cuda.empty_cache()
    check = _verdict(torch, dist, dev, rank, res, 1e-5)
    check["tokens"] = T_check * world
    del gx, gw, gi, gy
    # ---- timing
    fn = lambda i: layer.forward_prefill(x, weights=w, indices=idx)
    for i in range(W):
        fn(i)
    torch.cuda.synchronize()
    dist.barrier()
    with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        ms = timed_steps(torch, fn, K, 0, flush, stream)
        dist.barrier()
        torch.cuda.synchronize()
    st = torch.tensor([statistics.median(ms)], device=dev)
    dist.all_reduce(st, op=dist.ReduceOp.MAX)
    layer.track = True
    fn(0)
    layer.track = False
    pairs = torch.tensor([float(layer.local_active[-1])], device=dev)
    allp = [torch.zeros_like(pairs) for _ in range(world)]
    dist.all_gather(allp, pairs)
    step = float(st.item())
    f_routed = 2.0 * T * world * TOPK * 3 * I * D
    del layer
    torch.cuda.empty_cache()
    return {"config": "BASELINE.json configs[2]: T=8192 per GPU, Zipf(1.1) per rank (seed 7 + "
                      "rank), experts sharded %d per GPU, NCCL all-to-all dispatch/combine"
                      % (E // world),
            "metric": "MoE-layer prefill tok/s (a8, EP)", "unit": "tok/s",
            "value": round(T * world / (step / 1e3), 1), "ms": round(step, 4),
            "tokens_per_gpu": T, "n_gpus": world, "parallelism": "ep%d" % world,
            "experts_per_gpu": E // world, "scaling": "weak",
            "routed_tflops_job": round(f_routed / (step / 1e3) / 1e12, 1),
            "received_pairs_per_gpu": [int(v.item()) for v in allp],
            "clocks": clk.summary(), "ep_check": check}


def engram_ep_measure(q, torch, dist, dev, rank, world, K, W, flush, stream, peaks,
                      vocab=4_000_000, check_vocab=200_000):
    """d5 row-sharded (upstream ParallelEngramEmbedding layout): rank r holds rows
    [r * part, (r + 1) * part) of the table; every rank hashes the same T tokens.  Up to
    replicate_max_tokens every rank sums all tokens reading the peers' shards in place
    (one launch, no collective); above it each rank sums its slice of tokens from the
    shards in place and an all-gather assembles the result.  Total work is fixed as ranks
    are added ("strong").  ep_check: on a smaller table (same code path) the sharded result
    against rank 0's single-table result, bitwise."""
    import numpy as np
    hbm_peak, _, peak_src = peaks
    out = {}

    def shard_table(rows, seed_base):
        emb = q.engram.ParallelEngramEmbedding(rows, ENGRAM_DIM, block=ENGRAM_DIM)
        tab, sc = _engram_rows(torch, dev, emb.part, seed_base + rank)
        emb.weight, emb.scale = tab, sc
        return emb

    # ---- check on a small table
    args = _engram_args(check_vocab)
    primes, _ = q.engram.build_layout(args)
    rows = int(primes.sum())
    args.engram_num_embeddings = (rows,)
    hasher = q.engram.EngramHasher(args, np.arange(99092, dtype=np.int64), device=dev)
    emb = shard_table(rows, 900)
    gi = torch.Generator(device=dev).manual_seed(78)
    chk = {}
    for T in (1, 300):
        ids = torch.randint(0, 99092, (1, T), dtype=torch.int64, device=dev, generator=gi)
        cache = torch.zeros((1, T + 8), dtype=torch.int64, device=dev)
        y = hasher.lookup_sum(emb, ids, 0, cache)
        res = None
        if rank == 0:
            full = q.engram.EngramEmbedding(rows, ENGRAM_DIM, block=ENGRAM_DIM)
            parts = [_engram_rows(torch, dev, emb.part, 900 + r) for r in range(world)]
            full.weight = torch.cat([p[0] for p in parts])[:rows].contiguous()
            full.scale = torch.cat([p[1] for p in parts])[:rows].contiguous()
            del parts
            full.pack()
            c2 = torch.zeros_like(cache)
            yref = hasher.lookup_sum(full, ids, 0, c2)
            res = [float(torch.equal(yref, y)), _rel(y.float(), yref.float())]
            del full
            torch.cuda.empty_cache()
        chk[f"T{T}"] = _verdict(torch, dist, dev, rank, res, 0.0)
    check = {"bitwise": all(v["bitwise"] for v in chk.values()),
             "ok": all(v["ok"] for v in chk.values()), "table_rows": rows, "cases": chk}
    del emb
    torch.cuda.empty_cache()
    # ---- the BASELINE table
    args = _engram_args(vocab)
    primes, _ = q.engram.build_layout(args)
    rows = int(primes.sum())
    args.engram_num_embeddings = (rows,)
    hasher = q.engram.EngramHasher(args, np.arange(99092, dtype=np.int64), device=dev)
    emb = shard_table(rows, 55)
    gi = torch.Generator(device=dev).manual_seed(77)          # same ids on every rank
    for T in (1, PREFILL_T):
        start = 100 if T == 1 else 0
        ids = [torch.randint(0, 99092, (1, T), dtype=torch.int64, device=dev, generator=gi)
               for _ in range(8)]
        cache = torch.randint(0, 99092, (1, start + T + 8), dtype=torch.int64, device=dev,
                              generator=gi)

        def step(i, start=start):
            return hasher.lookup_sum(emb, ids[i % 8], start, cache)

        for i in range(W):
            step(i)
        torch.cuda.synchronize()
        dist.barrier()
        graphs = None
        if T <= emb.replicate_max_tokens:            # no collective: replay CUDA graphs
            graphs = graphed(torch, [lambda c=c: step(c) for c in range(8)])
            run = lambda i: graphs[i % 8].replay()
        else:
            run = step
        with Clocks(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
            ms = timed_steps(torch, run, K, 0 if graphs is None else 3, flush, stream)
            dist.barrier()
            torch.cuda.synchronize()
        del graphs
        st = torch.tensor([statistics.median(ms)], device=dev)
        dist.all_reduce(st, op=dist.ReduceOp.MAX)
        step_ms = float(st.item())
        byts = T * (ENGRAM_ROWS_PER_TOKEN * (ENGRAM_DIM + 1) + 2 * ENGRAM_DIM)
        out[f"engram_sharded_T{T}"] = {
            "config": f"BASELINE.json configs[4]: fp8 table [{rows} x 1024] + ue8m0 per row, "
                      f"row-sharded {emb.part} rows per GPU over {world} GPUs, T={T}",
            "metric": "engram hash + gather-sum tok/s (row-sharded table)", "unit": "tok/s",
            "value": round(T / (step_ms / 1e3), 1), "ms": round(step_ms, 4),
            "gbs_job": round(byts / (step_ms / 1e3) / 1e9, 1), "n_gpus": world,
            "parallelism": "rows%d" % world, "scaling": "strong", "table_rows": rows,
            "rows_per_gpu": emb.part, "peak_source": peak_src + " hbm_gbs",
            "clocks": clk.summary(), "ep_check": check}
    del emb
    torch.cuda.empty_cache()
    return out


def _engram_rows(torch, dev, n, seed):
    """One shard of the synthetic engram table: e4m3 codes uniform over non-NaN values,
    ue8m0 row scales in [115, 127] (the generator seeded per shard)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    tab = torch.empty((n, ENGRAM_DIM), dtype=torch.uint8, device=dev)
    for r0 in range(0, n, 1 << 20):
        c = tab[r0:r0 + (1 << 20)]
        c.random_(0, 254, generator=g)
        c += (c >= 127).to(torch.uint8)
    sc = torch.randint(115, 128, (n, 1), dtype=torch.uint8, device=dev, generator=g)
    return tab, sc


# ---------------------------------------------------------------- standalone modes --

def run_prefill_only(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        q = _package()
        rank = int(os.environ["RANK"])
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        r = prefill_ep_measure(q, torch, dist, dev, rank, world, args.steps, args.warmup, flush,
                               torch.cuda.current_stream(), _peaks(), T=args.prefill_tokens)
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(r))
        if not r["ep_check"]["ok"]:
            sys.exit(1)
        return
    q = _package()
    dev = torch.device("cuda", 0)
    layer = make_moe(q, torch, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    fn = prefill_a16_measurement if args.prefill_a16 else prefill_measurement
    with Clocks(0) as clk:
        r = fn(q, torch, dev, layer, flush, torch.cuda.current_stream(), _peaks(), args.steps,
               args.warmup, T=args.prefill_tokens, e2e=False)
    r["clocks"] = clk.summary()
    print(json.dumps(r))


def run_engram_only(args):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        q = _package()
        rank = int(os.environ["RANK"])
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=180))
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        r = engram_ep_measure(q, torch, dist, dev, rank, world, args.steps, args.warmup, flush,
                              torch.cuda.current_stream(), _peaks(), vocab=args.engram_vocab)
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            print(json.dumps(r))
        if not all(v["ep_check"]["ok"] for v in r.values()):
            sys.exit(1)
        return
    q = _package()
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with Clocks(0) as clk:
        r = engram_measurement(q, torch, dev, flush, torch.cuda.current_stream(), args.steps,
                               args.warmup, args.engram_vocab,
                               tokens=tuple(int(v) for v in args.engram_tokens.split(",")))
    r["clocks"] = clk.summary()
    print(json.dumps(r))


def run_affine_only(args):
    import torch
    q = _package()
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with Clocks(0) as clk:
        r = d4_measure(q, torch, dev, flush, torch.cuda.current_stream(), args.steps,
                       args.warmup, _peaks())
    r["clocks"] = clk.summary()
    print(json.dumps(r))


def run_gemv_only(args):
    import torch
    q = _package()
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with Clocks(0) as clk:
        r = d1_measure(q, torch, dev, flush, torch.cuda.current_stream(), args.steps,
                       args.warmup, _peaks(), tuple(int(v) for v in args.gemv_m.split(",")))
    r["clocks"] = clk.summary()
    print(json.dumps(r))


# ---------------------------------------------------------------- CPU baselines --
# The numpy port of the reference's algorithm (oracle/, restating deepseek_v41_mlx/
# dequant.py, moe.py, engram.py and the MLX affine format) timed on the host cores.  The
# oracle is the checker of the tests; here it is only the baseline beside the GPU numbers.

def _oracle():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import engram as OE
    from oracle import formats as F
    from oracle import linear as OL
    from oracle import moe as OM
    return F, OM, OL, OE


def cpu_moe_setup(seed=0):
    """Inputs of one T=64 decode step and the release-layout weights of the experts it
    routes to (generated outside any timing)."""
    import numpy as np
    F, OM, _, _ = _oracle()
    rng = np.random.default_rng(seed)
    x = F.bf16_bits_to_f32(F.f32_to_bf16_bits(rng.standard_normal((T_HEAD, D)).astype(np.float32)))
    gw = F.bf16_bits_to_f32(F.f32_to_bf16_bits(
        (rng.standard_normal((E, D)) * D ** -0.5).astype(np.float32)))
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    _, idx, _ = OM.gate(x, gw, bias, TOPK, acc=np.float32)

    def fp4(n, k):
        return (rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8),
                rng.integers(120, 129, size=(n, k // 32), dtype=np.uint8))

    def fp8(n, k):
        w = rng.integers(0, 256, size=(n, k), dtype=np.uint8)
        w[(w & 0x7F) == 0x7F] = 0
        return w, rng.integers(118, 128, size=(n // 32, k // 32), dtype=np.uint8)

    experts = {int(e): (fp4(I, D), fp4(I, D), fp4(D, I)) for e in np.unique(idx)}
    shared = (fp8(I, D), fp8(I, D), fp8(D, I))
    return {"x": x, "gw": gw, "bias": bias, "experts": experts, "shared": shared}


def cpu_moe_step(ctx, pool):
    """One whole MoE decode step of the port (moe.py:105-112): router, every routed expert
    the batch reaches (dequant_fp4 + SwitchGLU, one task per expert on the thread pool),
    the shared expert, the fp32 combine in top-k order.  -> seconds."""
    import numpy as np
    F, OM, _, _ = _oracle()
    x = ctx["x"]
    t0 = time.perf_counter()
    w, idx, _ = OM.gate(x, ctx["gw"], ctx["bias"], TOPK, acc=np.float32)

    def expert(e):
        t_sel, j_sel = np.nonzero(idx == e)
        (w1, s1), (w3, s3), (w2, s2) = ctx["experts"][e]
        return t_sel, j_sel, OM.expert_fp4(x[t_sel], w1, s1, w3, s3, w2, s2, 10.0, True,
                                           np.float32)

    def shared():
        (a, sa), (b, sb), (c, scc) = ctx["shared"]
        return OM.shared_expert_fp8(x, a, sa, b, sb, c, scc, 10.0, True, np.float32)

    fut_sh = pool.submit(shared)
    ys = np.zeros((T_HEAD, TOPK, D), dtype=np.float32)
    for t_sel, j_sel, ye in pool.map(expert, [int(e) for e in np.unique(idx)]):
        ys[t_sel, j_sel] = ye
    y = np.zeros((T_HEAD, D), dtype=np.float32)
    for j in range(TOPK):
        y = (y + ys[:, j] * w[:, j:j + 1]).astype(np.float32)
    y = (y + fut_sh.result()).astype(np.float32)
    F.round_bf16(y)
    return time.perf_counter() - t0


def cpu_moe_baseline():
    """cpu_baseline of the headline: one whole T=64 step of the port on the host cores."""
    from concurrent.futures import ThreadPoolExecutor
    cores = os.cpu_count()
    ctx = cpu_moe_setup()
    with ThreadPoolExecutor(cores) as pool:
        s = cpu_moe_step(ctx, pool)
    n = len(ctx["experts"])
    del ctx
    return {"value": round(T_HEAD / s, 4), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"one whole T=64 step: router, all {n} routed experts the batch reaches "
                      f"(a thread-pool task each), shared expert, combine (numpy fp32)",
            "step_s": round(s, 3), "estimated": False}


def _median_time(fn, n=3, budget=None):
    ts = []
    for _ in range(n):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
        if budget and sum(ts) > budget:
            break
    return statistics.median(ts)


def cpu_sub_baselines(sub, seconds):
    """cpu_baseline of each sub-measurement, in its own unit (bounded samples, stated)."""
    import numpy as np
    F, OM, OL, OE = _oracle()
    cores = os.cpu_count()
    rng = np.random.default_rng(5)
    base = {"cores": cores, "kind": "port"}
    # d1: dequant_fp8 then matmul at full size
    w = rng.integers(0, 256, size=(D1_N, D1_K), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0
    s = rng.integers(118, 128, size=(D1_N // 32, D1_K // 32), dtype=np.uint8)
    for M in (1, 32):
        key = f"gemv_fp8_block_M{M}"
        if key not in sub:
            continue
        x = rng.standard_normal((M, D1_K)).astype(np.float32)
        byts = D1_N * D1_K + (D1_N // 32) * (D1_K // 32) + M * D1_K * 2 + M * D1_N * 2
        t = _median_time(lambda: x @ F.dequant_fp8(w, s, "f32").T)
        sub[key]["cpu_baseline"] = dict(base, value=round(byts / t / 1e9, 3), unit="GB/s",
                                        sample=f"full size: dequant_fp8 + fp32 matmul, median "
                                               f"of 3 ({t * 1e3:.1f} ms)")
    # d4: mx.dequantize then matmul at full size (bf16 weights, fp32 BLAS)
    for bits in (4, 8):
        wq = rng.integers(0, 2 ** 32, size=(D4_N, D4_K * bits // 32), dtype=np.uint64).astype(np.uint32)
        sc = F.f32_to_bf16_bits(rng.uniform(0.001, 0.02, size=(D4_N, D4_K // 64)).astype(np.float32))
        bi = F.f32_to_bf16_bits((rng.standard_normal((D4_N, D4_K // 64)) * 0.05).astype(np.float32))
        for M in (1, 16, 4096):
            key = f"affine{bits}_M{M}"
            if key not in sub:
                continue
            x = rng.standard_normal((M, D4_K)).astype(np.float32)

            def run():
                wd = F.bf16_bits_to_f32(F.dequant_affine(wq, sc, bi, bits, 64, D4_K))
                return x @ wd.T
            t = _median_time(run, n=1)
            if M <= 16:
                byts = D4_N * D4_K * bits // 8 + 2 * D4_N * (D4_K // 64) * 2 + M * D4_K * 2 + M * D4_N * 2
                v, u = byts / t / 1e9, "GB/s"
            else:
                v, u = 2.0 * M * D4_N * D4_K / t / 1e12, "TFLOP/s"
            sub[key]["cpu_baseline"] = dict(base, value=round(v, 4), unit=u,
                                            sample=f"full size: dequant_affine -> bf16 -> fp32 "
                                                   f"matmul ({t:.2f} s)")
    # d3: prefill in a8 numerics; a sample of experts timed, scaled (stated)
    if "moe_prefill_T8192_a8" in sub:
        est = cpu_prefill_estimate(sub["moe_prefill_T8192_a8"], seconds)
        sub["moe_prefill_T8192_a8"]["cpu_baseline"] = dict(base, **est)
        if "moe_prefill_T8192_a16" in sub:
            # the port's CPU path has the same weight decode and the same products (bf16
            # activations, no act_quant), so the sampled costs carry over
            sub["moe_prefill_T8192_a16"]["cpu_baseline"] = dict(
                base, **est, note="the a8 sample's decode and product costs (the port decodes "
                                  "the same weights and multiplies the same shapes)")
    # d5: hash + gather + dequant + sum on a host table (the BASELINE table does not fit)
    for T in (1, PREFILL_T):
        key = f"engram_T{T}"
        if key in sub:
            sub[key]["cpu_baseline"] = dict(base, **cpu_engram(T))


def cpu_prefill_estimate(meas, seconds, n_sample=6):
    """The a8 prefill layer of the oracle (upstream model.py:889-904 with fp4 experts) on a
    sample of experts with the pair counts of the measured Zipf routing: per expert, the
    weight decode (once) and the gate/up/down products of its pairs; scaled to every active
    expert and pair; the shared expert and act_quant on 512 tokens, scaled to 8192."""
    import numpy as np
    F, OM, OL, _ = _oracle()
    rng = np.random.default_rng(9)
    T = meas["tokens"]
    n_active = meas["experts_active"]
    P = T * TOPK
    counts = np.linspace(meas["pairs_min_expert"], min(meas["pairs_max_expert"], 2048),
                         n_sample).astype(int)
    t_dec, t_mm, pairs = 0.0, 0.0, 0
    for n in counts:
        w1, s1 = rng.integers(0, 256, (I, D // 2), dtype=np.uint8), rng.integers(120, 129, (I, D // 32), dtype=np.uint8)
        w3, s3 = rng.integers(0, 256, (I, D // 2), dtype=np.uint8), rng.integers(120, 129, (I, D // 32), dtype=np.uint8)
        w2, s2 = rng.integers(0, 256, (D, I // 2), dtype=np.uint8), rng.integers(120, 129, (D, I // 32), dtype=np.uint8)
        x = F.round_bf16(rng.standard_normal((int(n), D)).astype(np.float32))
        t0 = time.perf_counter()
        W1, W3, W2 = (F.dequant_fp4(a, b, "f32") for a, b in ((w1, s1), (w3, s3), (w2, s2)))
        t1 = time.perf_counter()
        xq = OL.act_dequant(x)
        g = F.round_bf16(xq @ W1.T)
        u = F.round_bf16(xq @ W3.T)
        h = F.round_bf16(np.clip(u, -10, 10) * (np.minimum(g, 10) / (1 + np.exp(-np.minimum(g, 10)))))
        F.round_bf16(OL.act_dequant(h) @ W2.T)
        t2 = time.perf_counter()
        t_dec += t1 - t0
        t_mm += t2 - t1
        pairs += int(n)
        if t_dec + t_mm > seconds:
            break
    done = max(1, len(counts) if t_dec + t_mm <= seconds else list(counts).index(n) + 1)
    xs = F.round_bf16(rng.standard_normal((512, D)).astype(np.float32))
    sw = [rng.integers(0, 256, (n, k), dtype=np.uint8) for n, k in ((I, D), (I, D), (D, I))]
    for a in sw:
        a[(a & 0x7F) == 0x7F] = 0
    ss = [rng.integers(118, 128, (n // 32, k // 32), dtype=np.uint8) for n, k in ((I, D), (I, D), (D, I))]
    t0 = time.perf_counter()
    xq = OL.act_dequant(xs)
    W = [F.dequant_fp8(a, b, "f32") for a, b in zip(sw, ss)]
    g = F.round_bf16(xq @ W[0].T)
    u = F.round_bf16(xq @ W[1].T)
    h = F.round_bf16(np.clip(u, -10, 10) * (np.minimum(g, 10) / (1 + np.exp(-np.minimum(g, 10)))))
    F.round_bf16(OL.act_dequant(h) @ W[2].T)
    t_sh = (time.perf_counter() - t0) * (T / 512)
    est = n_active * (t_dec / done) + P * (t_mm / pairs) + t_sh
    return {"value": round(T / est, 2), "unit": "tok/s", "estimated": True,
            "sample": f"{done} experts timed (pair counts {list(map(int, counts[:done]))} of the "
                      f"Zipf routing): fp4 decode {t_dec / done:.2f} s/expert, a8 products "
                      f"{t_mm / pairs * 1e3:.2f} ms/pair; scaled to {n_active} experts and {P} "
                      f"pairs; shared expert on 512 tokens x16 (numpy fp32)",
            "est_step_s": round(est, 2)}


def cpu_engram(T, vocab=40_000):
    """hash + gather + dequant + fp32 sum of the oracle (engram.py:154-203) on a host table of
    ~1M rows with the BASELINE row format (the 98 GB table does not fit in host memory;
    a random row read costs the same from either)."""
    import types
    import numpy as np
    F, _, _, OE = _oracle()
    args = types.SimpleNamespace(engram_layer_ids=(1,), engram_max_ngram_size=4,
                                 engram_vocab_size=vocab, engram_n_heads=8, engram_pad_id=2)
    primes, offsets = OE.build_layout(1, 4, 8, vocab)
    rows = int(primes.sum())
    mult = OE.compute_hash_multipliers((1,), 4, 99092)
    rng = np.random.default_rng(3)
    table = np.frombuffer(rng.bytes(rows * ENGRAM_DIM), np.uint8).reshape(rows, ENGRAM_DIM).copy()
    table[(table & 0x7F) == 0x7F] = 0
    scale = rng.integers(115, 128, (rows, 1), dtype=np.uint8)
    ids = rng.integers(0, 99092, (1, T))
    tm = np.arange(99092, dtype=np.int64)
    cache = np.zeros((1, T + 8), dtype=np.int64)

    def run():
        idx = OE.engram_hash(ids, 0, cache, tm, mult, primes, offsets, 2, 4)
        return OE.gather_sum(table, scale, idx[0, :, 0], ENGRAM_DIM)
    t = _median_time(run, n=3)
    del args
    return {"value": round(T / t, 2), "unit": "tok/s", "estimated": False,
            "sample": f"T={T} through the oracle's hash and gather-sum on a {rows}-row host "
                      f"table ({t * 1e3:.1f} ms; the 98 GB table does not fit in host memory)"}


def run_reference(args):
    """The reference arm: the port's whole T=64 decode step on the host cores (all threads),
    as many whole steps as fit the time budget after one warm-up step."""
    from concurrent.futures import ThreadPoolExecutor
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count()
    t_start = time.perf_counter()
    ctx = cpu_moe_setup()
    times = []
    with ThreadPoolExecutor(cores) as pool:
        warm = cpu_moe_step(ctx, pool) if args.warmup > 0 else None
        while len(times) < max(1, args.steps):
            times.append(cpu_moe_step(ctx, pool))
            if time.perf_counter() - t_start > args.ref_budget_s:
                break
    wall = time.perf_counter() - t_start
    st = statistics.mean(times)
    v = round(T_HEAD / st, 4)
    n = len(ctx["experts"])
    cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
           "sample": f"whole T=64 steps: router, all {n} routed experts the batch reaches (a "
                     f"thread-pool task each), shared expert, combine (numpy fp32)",
           "estimated": False}
    print(json.dumps({
        "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world, "steps": len(times),
        "steps_requested": args.steps, "warmup": 1 if warm is not None else 0,
        "ms_per_step": round(st * 1e3, 2), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (numpy)", "impl": "reference", "estimated": False,
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
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="budget of each sampled CPU baseline")
    ap.add_argument("--ref-budget-s", type=float, default=150.0,
                    help="wall-time budget of the reference arm (whole steps)")
    ap.add_argument("--experts", type=int, default=384,
                    help="routed experts (384 = BASELINE; smaller only for ncu captures)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only the T=8192 a8 prefill measurement (one JSON line)")
    ap.add_argument("--prefill-tokens", type=int, default=PREFILL_T)
    ap.add_argument("--prefill-a16", action="store_true",
                    help="with --prefill-only: the port's numerics (MoE.prefill_a16)")
    ap.add_argument("--affine-only", action="store_true",
                    help="only the affine (d4) measurements (one JSON line)")
    ap.add_argument("--gemv-only", action="store_true",
                    help="only the fp8 dense GEMV (d1) measurements (one JSON line)")
    ap.add_argument("--engram-only", action="store_true",
                    help="only the engram d5 measurement (one JSON line)")
    ap.add_argument("--engram-tokens", default="1,8192",
                    help="engram positions a step (comma list; only with --engram-only)")
    ap.add_argument("--gemv-m", default="1,32",
                    help="activation rows of the d1 GEMV (comma list; only with --gemv-only)")
    ap.add_argument("--engram-vocab", type=int, default=4_000_000,
                    help="engram_vocab_size of d5 (4,000,000 = BASELINE; smaller only for ncu "
                         "captures)")
    args = ap.parse_args()
    global E, ROUTER_BYTES
    E = args.experts
    ROUTER_BYTES = E * D * 2
    if args.prefill_only:
        run_prefill_only(args)
    elif args.engram_only:
        run_engram_only(args)
    elif args.affine_only:
        run_affine_only(args)
    elif args.gemv_only:
        run_gemv_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
