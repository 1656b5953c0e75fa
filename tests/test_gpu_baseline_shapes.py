"""Parity at the BASELINE.json shapes, on the exact paths bench.py times.

The layer is ``bench.make_moe`` (384 fp4 experts, dim 7168, moe_inter_dim 2048,
top-6, fp8 shared expert, the release layout with the bench's seeded values) and
the routing of the prefill case is ``bench.zipf_routing`` (BASELINE.json
Zipf(1.1) over a seeded expert permutation).  Every token of a batch
goes through the device path; the CPU oracle then recomputes a seeded sample of
tokens (each token's output depends only on its own row and routing), which keeps
the oracle's fp4 decode of the sampled tokens' experts affordable.

* decode, T=64 (configs[1], the headline): the public ``MoE.__call__`` default --
  CUDA-graph replay, decode-packed scales, the row-pair down projection, the split-K
  counts of ~250 active experts -- against ``oracle.moe.moe_forward`` on the kernel's
  routing: 1e-5 with fp32 output (exact mode) and 1e-2 with bf16 output (port mode).
  Reference: deepseek_v41_mlx/moe.py:105-112.
* prefill, T=8192: ``MoE.prefill_a8`` (act_quant + tcgen05 block-scaled
  grouped GEMMs, wide and narrow tiles) against ``oracle.moe.moe_forward_upstream_a8``
  on the same routing, 1e-2 (upstream a8 numerics differ from the oracle only in the
  accumulation order).  Reference: docs/reference/model.py:889-904.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
import deepseek_v41_mlx_b200 as q
from conftest import rel_fro
from deepseek_v41_mlx_b200 import _lib as L
from oracle import formats as F
from oracle import moe as OM

pytestmark = pytest.mark.gpu

E, D, I, K = bench.E, bench.D, bench.I, bench.TOPK
CFG = dict(topk=K, score_func="sqrtsoftplus", gate_temp=1.0, norm_topk_prob=True,
           route_scale=1.5, swiglu_limit=10.0)


@pytest.fixture(scope="module")
def layer(cuda):
    m = bench.make_moe(q, torch, torch.device("cuda", 0))
    yield m
    del m
    torch.cuda.empty_cache()


def _oracle_params(m, experts):
    """numpy copies of the weights the oracle needs: the given routed experts and the
    shared expert; the router weights as fp32 values of the bf16 tensor."""
    p = {k: {} for k in ("w1", "s1", "w3", "s3", "w2", "s2")}
    for e in experts:
        for key, proj in (("1", m.experts.gate_proj), ("3", m.experts.up_proj),
                          ("2", m.experts.down_proj)):
            p["w" + key][int(e)] = proj.weight[int(e)].cpu().numpy()
            p["s" + key][int(e)] = proj.scales[int(e)].cpu().numpy()
    for key in ("1", "2", "3"):
        pr = getattr(m.shared_experts, "w" + key)
        p["sw" + key] = pr.weight.cpu().numpy()
        p["ss" + key] = pr.scales.cpu().numpy()
    p["gate_w"] = m.gate.weight.float().cpu().numpy()
    p["gate_bias"] = m.gate.bias.float().cpu().numpy()
    return p


def _bf16_values(x):
    return x.float().cpu().numpy()


def test_decode_headline_T64(layer):
    T = bench.T_HEAD
    g = torch.Generator(device="cuda").manual_seed(6464)
    x = torch.randn(T, D, device="cuda", generator=g).to(torch.bfloat16)
    xf = _bf16_values(x)
    rng = np.random.default_rng(64)
    sample = np.sort(rng.choice(T, 10, replace=False))
    results = {}
    for exact in (True, False):
        layer.round_bf16 = not exact
        odt = torch.float32 if exact else torch.bfloat16
        y, w, idx = layer(x, with_routing=True, out_dtype=odt)
        assert layer.cuda_graph and layer._dpack is not None      # the bench's path
        results[exact] = (y, w, idx)
        w_np, idx_np = w.cpu().numpy(), idx.cpu().numpy()
        gw, gb = layer.gate.weight.float().cpu().numpy(), layer.gate.bias.cpu().numpy()
        gap = OM.topk_margin(xf, gw, gb, K)
        ow, oidx, _ = OM.gate(xf, gw, gb, K)
        ok = gap > 1e-5
        assert ok.mean() > 0.9
        assert np.array_equal(idx_np[ok], oidx[ok])
        np.testing.assert_allclose(w_np[ok], ow[ok], rtol=1e-5, atol=1e-7)
        assert len(np.unique(idx_np)) > 200                        # ~250 active experts
        p = _oracle_params(layer, np.unique(idx_np[sample]))
        want, _, _ = OM.moe_forward(xf[sample], p, CFG, round_bf16_io=not exact,
                                    routing=(w_np[sample], idx_np[sample]))
        got = y.float().cpu().numpy()[sample]
        assert rel_fro(got, want) < (1e-5 if exact else 1e-2), "exact" if exact else "port"
    # direct launches (no graph) run the row-pair down projection and give the same bits
    layer.round_bf16 = True
    layer.cuda_graph = False
    try:
        L.prof_enable(True)
        y2, w2, idx2 = layer(x, with_routing=True, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        names = set(L.prof_report())
    finally:
        L.prof_enable(False)
        layer.cuda_graph = True
    assert "moe_expert_down_fp4_pairs" in names and "moe_expert_gate_up_fp4" in names
    y, w, idx = results[False]
    assert torch.equal(idx2, idx) and torch.equal(w2, w) and torch.equal(y2, y)


def test_prefill_a8_d3_shape(layer):
    T = 8192
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4321)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = bench.zipf_routing(torch, dev, x, layer.gate.weight, T)
    L.prof_enable(True)
    try:
        y = layer.prefill_a8(x, weights=w, indices=idx, out_dtype=torch.float32)
        torch.cuda.synchronize()
        names = set(L.prof_report())
    finally:
        L.prof_enable(False)
    # the tile mix the bench times: heavy experts on wide tiles, light ones on narrow tiles
    assert {"pf_gate_up_fp4", "pf_gate_up_fp4_narrow", "pf_down_fp4",
            "pf_down_fp4_narrow"} <= names
    w_np, idx_np = w.cpu().numpy(), idx.cpu().numpy()
    counts = np.bincount(idx_np.reshape(-1), minlength=E)
    assert counts.max() > 2000 and (counts > 0).sum() > 300       # Zipf-skewed, most active
    rng = np.random.default_rng(8192)
    light = np.nonzero((counts[idx_np] <= 64).any(-1))[0]          # tokens on narrow tiles
    sample = np.unique(np.concatenate([rng.choice(T, 12, replace=False),
                                       rng.choice(light, 12, replace=False)]))
    xf = _bf16_values(x[torch.from_numpy(sample).to(dev)])
    p = _oracle_params(layer, np.unique(idx_np[sample]))
    want, _, _ = OM.moe_forward_upstream_a8(F.round_bf16(xf), p, CFG,
                                            routing=(w_np[sample], idx_np[sample]))
    got = y.cpu().numpy()[sample]
    assert rel_fro(got, want) < 1e-2


def test_prefill_a16_d3_shape(layer):
    """BASELINE configs[2] in the port's numerics on the tensor cores (MoE.prefill_a16):
    exact mode, fp32 output, against oracle.moe.moe_forward (float64 accumulation) on
    sampled tokens.  The tensor cores accumulate a tile's whole K (7168 for gate/up, 2 x 2048
    for the hi + lo down projection) in one fp32 accumulator, whose rounding grows with the
    number of MMA steps: measured 8.4e-5 here (the small shapes of test_gpu_prefill_a16.py,
    K <= 512, stay under 1e-5; the decode engine, which sums per-32 partials, meets 1e-5 at
    this shape).  Bound: 2e-4."""
    T = 8192
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4322)
    x = torch.randn(T, D, device=dev, generator=g).to(torch.bfloat16)
    w, idx = bench.zipf_routing(torch, dev, x, layer.gate.weight, T)
    layer.round_bf16 = False
    try:
        y = layer.prefill_a16(x, weights=w, indices=idx, out_dtype=torch.float32)
        torch.cuda.synchronize()
    finally:
        layer.round_bf16 = True
    w_np, idx_np = w.cpu().numpy(), idx.cpu().numpy()
    counts = np.bincount(idx_np.reshape(-1), minlength=E)
    rng = np.random.default_rng(8193)
    light = np.nonzero((counts[idx_np] <= 64).any(-1))[0]
    sample = np.unique(np.concatenate([rng.choice(T, 12, replace=False),
                                       rng.choice(light, 12, replace=False)]))
    xf = _bf16_values(x[torch.from_numpy(sample).to(dev)])
    p = _oracle_params(layer, np.unique(idx_np[sample]))
    want, _, _ = OM.moe_forward(xf, p, CFG, round_bf16_io=False,
                                routing=(w_np[sample], idx_np[sample]))
    assert rel_fro(y.cpu().numpy()[sample], want) < 2e-4
