"""MoE router, routed experts and the decode layer vs the oracle (port semantics).

Routing: the selected expert sets must match the oracle for every token whose
k-th / (k+1)-th biased-score gap exceeds 1e-5 (fp32 accumulation order may flip
closer ties); weights within 1e-5 relative.  Layer outputs are compared using
the kernel's own routing so that expert math is checked independently:
1e-5 (fp32 out, exact mode) and 1e-2 (bf16 out, port rounding).
"""

from __future__ import annotations

import ctypes as C
import types

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import golden, rel_fro
from deepseek_v41_mlx_b200 import _lib as L
from gen import bf16_acts, moe_params
from oracle import moe as OM

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bf(bits):
    return _d(bits.view(np.int16)).view(torch.bfloat16)


def _args(E, D, I, k, limit=10.0):
    return types.SimpleNamespace(n_activated_experts=k, score_func="sqrtsoftplus", gate_temp=1.0,
                                 norm_topk_prob=True, route_scale=1.5, n_routed_experts=E, dim=D,
                                 moe_inter_dim=I, swiglu_limit=limit)


def _moe(p, args, round_bf16):
    m = q.moe.MoE(args, round_bf16=round_bf16)
    m.gate.weight = _bf(p["gate_w_bits"])
    m.gate.bias = _d(p["gate_bias"])
    for name, key in (("gate_proj", "1"), ("up_proj", "3"), ("down_proj", "2")):
        getattr(m.experts, name).weight = _d(p["w" + key])
        getattr(m.experts, name).scales = _d(p["s" + key])
    for key in ("1", "2", "3"):
        getattr(m.shared_experts, "w" + key).weight = _d(p["sw" + key])
        getattr(m.shared_experts, "w" + key).scales = _d(p["ss" + key])
    return m


def _cfg(args):
    return dict(topk=args.n_activated_experts, score_func="sqrtsoftplus", gate_temp=1.0,
                norm_topk_prob=True, route_scale=1.5, swiglu_limit=args.swiglu_limit)


def _check_routing(x, p, args, w, idx, margin=1e-5):
    ow, oidx, _ = OM.gate(x, p["gate_w"], p["gate_bias"], args.n_activated_experts)
    gap = OM.topk_margin(x, p["gate_w"], p["gate_bias"], args.n_activated_experts)
    ok = gap > margin
    assert ok.mean() > 0.9
    assert np.array_equal(np.sort(idx[ok], -1), np.sort(oidx[ok], -1))
    assert np.array_equal(idx[ok], oidx[ok])          # descending order too
    np.testing.assert_allclose(w[ok], ow[ok], rtol=1e-5, atol=1e-7)


def test_router_golden(cuda):
    g = golden("router_expert.npz")
    args = _args(g["gate_w"].shape[0], g["gate_w"].shape[1], 64, int(g["topk"]))
    gate = q.moe.Gate(args)
    gate.weight = _d(g["gate_w"]).to(torch.bfloat16)
    gate.bias = _d(g["gate_bias"])
    w, idx = gate(_d(g["x"]).to(torch.bfloat16))
    assert np.array_equal(np.sort(idx.cpu().numpy(), -1), np.sort(g["indices"], -1))
    np.testing.assert_allclose(np.sort(w.cpu().numpy(), -1), np.sort(g["weights"], -1),
                               rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("T", [1, 8, 64])
def test_router_baseline_shape(cuda, T):
    rng = np.random.default_rng(T)
    E, D, k = 384, 7168, 6
    gwb, gw = bf16_acts(rng, E, D, std=D ** -0.5)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    xb, xf = bf16_acts(rng, T, D)
    args = _args(E, D, 2048, k)
    gate = q.moe.Gate(args)
    gate.weight, gate.bias = _bf(gwb), _d(bias)
    w, idx = gate(_bf(xb))
    _check_routing(xf, {"gate_w": gw, "gate_bias": bias}, args, w.cpu().numpy(),
                   idx.cpu().numpy())


def test_experts_vs_golden_expert(cuda):
    """SwitchGLU path on the upstream Expert golden (fp32, exact mode)."""
    g = golden("router_expert.npz")
    E, D = g["gate_w"].shape
    I = g["w1"].shape[1]
    args = _args(E, D, I, int(g["topk"]))
    p = {k: g[k] for k in ("w1", "s1", "w3", "s3", "w2", "s2", "sw1", "ss1", "sw3", "ss3",
                           "sw2", "ss2", "gate_bias")}
    p["gate_w_bits"] = np.zeros((E, D), np.uint16)
    m = _moe(p, args, round_bf16=False)
    e0 = int(g["e0"])
    x = _d(g["x"][:5]).to(torch.bfloat16)
    idx = torch.full((5, 1), e0, dtype=torch.int32, device="cuda")
    m.args = _args(E, D, I, 1)
    y = m.experts(x, idx)[:, 0].cpu().numpy()
    assert rel_fro(y, g["y_expert"]) < 1e-5


@pytest.mark.parametrize("T", [1, 5, 33])
def test_moe_decode_small(cuda, T):
    rng = np.random.default_rng(100 + T)
    E, D, I, k = 16, 256, 128, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    for exact in (True, False):
        m = _moe(p, args, round_bf16=not exact)
        y, w, idx = m(_bf(xb), with_routing=True, out_dtype=torch.float32 if exact else torch.bfloat16)
        w, idx = w.cpu().numpy(), idx.cpu().numpy()
        _check_routing(xf, p, args, w, idx)
        want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=not exact, routing=(w, idx))
        tol = 1e-5 if exact else 1e-2
        assert rel_fro(y.float().cpu().numpy(), want) < tol


def test_moe_experts_matches_decode(cuda):
    """MoE.experts(xf, indices) (unweighted [T, k, D]) recombines to the layer output."""
    rng = np.random.default_rng(7)
    E, D, I, k, T = 16, 256, 128, 4, 9
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    m = _moe(p, args, round_bf16=False)
    y, w, idx = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
    ye = m.experts(_bf(xb), idx)
    want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=False, with_shared=False,
                                routing=(w.cpu().numpy(), idx.cpu().numpy()))
    got = (ye * w[..., None]).sum(1).cpu().numpy()
    assert rel_fro(got, want) < 1e-5


@pytest.mark.parametrize("T", [1, 8])
def test_moe_decode_baseline_shape(cuda, T):
    """config 2: 384 experts, D 7168, I 2048, top-6; oracle on the selected experts."""
    E, D, I, k = 384, 7168, 2048, 6
    g = torch.Generator(device="cuda").manual_seed(T)
    rng = np.random.default_rng(T)
    W = {}
    for name, shp in (("w1", (E, I, D // 2)), ("w3", (E, I, D // 2)), ("w2", (E, D, I // 2))):
        W[name] = torch.randint(0, 256, shp, dtype=torch.uint8, device="cuda", generator=g)
        W["s" + name[1]] = torch.randint(120, 129, shp[:2] + (shp[2] * 2 // 32,), dtype=torch.uint8,
                                         device="cuda", generator=g)
    sh = {}
    for name, (n, kk) in (("sw1", (I, D)), ("sw3", (I, D)), ("sw2", (D, I))):
        wv = torch.randint(0, 256, (n, kk), dtype=torch.uint8, device="cuda", generator=g)
        wv[(wv & 0x7F) == 0x7F] = 0
        sh[name] = wv
        sh["ss" + name[2]] = torch.randint(118, 128, (n // 32, kk // 32), dtype=torch.uint8,
                                           device="cuda", generator=g)
    gwb, gw = bf16_acts(rng, E, D, std=D ** -0.5)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    xb, xf = bf16_acts(rng, T, D)
    args = _args(E, D, I, k)
    m = q.moe.MoE(args, round_bf16=False)
    m.gate.weight, m.gate.bias = _bf(gwb), _d(bias)
    for name, key in (("gate_proj", "1"), ("up_proj", "3"), ("down_proj", "2")):
        getattr(m.experts, name).weight = W["w" + key]
        getattr(m.experts, name).scales = W["s" + key]
    for key in ("1", "2", "3"):
        getattr(m.shared_experts, "w" + key).weight = sh["sw" + key]
        getattr(m.shared_experts, "w" + key).scales = sh["ss" + key]
    y, w, idx = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
    w, idx = w.cpu().numpy(), idx.cpu().numpy()
    _check_routing(xf, {"gate_w": gw, "gate_bias": bias}, args, w, idx)
    used = np.unique(idx)
    p = {"w1": {}, "s1": {}, "w3": {}, "s3": {}, "w2": {}, "s2": {}}
    for e in used:
        for key in p:
            p[key][e] = W[key][e].cpu().numpy()
    for key in sh:
        p[key] = sh[key].cpu().numpy()
    want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=False, routing=(w, idx))
    assert rel_fro(y.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("T", [1, 6, 40])
def test_moe_graph_replay_matches_direct(cuda, T):
    """CUDA-graph replay (shared expert on the forked stream) == direct launches, bitwise,
    for several inputs through one captured graph; replacing a weight re-captures."""
    rng = np.random.default_rng(40 + T)
    E, D, I, k = 16, 256, 128, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    mg = _moe(p, args, round_bf16=True)
    md = _moe(p, args, round_bf16=True)
    md.cuda_graph = False
    for _ in range(3):
        xb, _ = bf16_acts(rng, T, D)
        a, wa, ia = mg(_bf(xb), with_routing=True)
        b, wb, ib = md(_bf(xb), with_routing=True)
        assert torch.equal(a, b) and torch.equal(wa, wb) and torch.equal(ia, ib)
    p2 = moe_params(np.random.default_rng(1), E, D, I)
    mg.shared_experts.w2.weight = _d(p2["sw2"])
    md.shared_experts.w2.weight = mg.shared_experts.w2.weight
    xb, _ = bf16_acts(rng, T, D)
    assert torch.equal(mg(_bf(xb)), md(_bf(xb)))


def test_moe_decode_capi_workspace_reuse(cuda):
    """Two calls sharing one workspace give identical bits (no stale state)."""
    rng = np.random.default_rng(3)
    E, D, I, k, T = 16, 256, 128, 4, 12
    p = moe_params(rng, E, D, I)
    m = _moe(p, _args(E, D, I, k), round_bf16=True)
    xb, _ = bf16_acts(rng, T, D)
    a = m(_bf(xb))
    b = m(_bf(xb))
    assert torch.equal(a, b)
    st = C.c_uint32(0)
    L.call("dsv41_device_status", torch.cuda.current_stream().cuda_stream, C.byref(st))
    assert st.value == 0


@pytest.mark.parametrize("T", [1, 7, 40])
def test_moe_decode_packed_scales_identical(cuda, T):
    """Decode with the routed scales in the decode-packed layout (one contiguous block per
    64-row tile and stage) gives the same bits as the release layout, graph and direct."""
    rng = np.random.default_rng(300 + T)
    E, D, I, k = 12, 512, 256, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, _ = bf16_acts(rng, T, D)
    outs = []
    for pack in (False, True):
        for graph in (False, True):
            m = _moe(p, args, round_bf16=True)
            m.pack_decode_scales, m.cuda_graph = pack, graph
            y, w, idx = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
            ye = m.experts(_bf(xb), idx)
            outs.append((y, w, idx, ye))
            assert (m._dpack is not None) == pack
    for y, w, idx, ye in outs[1:]:
        assert torch.equal(y, outs[0][0]) and torch.equal(idx, outs[0][2])
        assert torch.equal(ye, outs[0][3])


def test_moe_decode_pack_rejected_by_prefill(cuda):
    """The prefill entries read the release layout and refuse the packed-scales flag."""
    rng = np.random.default_rng(4)
    E, D, I, k = 8, 256, 256, 2
    p = moe_params(rng, E, D, I)
    m = _moe(p, _args(E, D, I, k), round_bf16=True)
    cfg, W = m._decode_args()
    assert cfg.flags & L.MOE_PACKED_SCALES
    x = torch.zeros(4, D, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(4, D, dtype=torch.float32, device="cuda")
    ws = L.workspace(L.load().dsv41_moe_prefill_workspace_size(C.byref(cfg), 4, 0, 0), "cuda")
    st = L.load().dsv41_moe_prefill(C.byref(cfg), C.byref(W), None, L.ptr(x), 4, None, None,
                                    L.dtype_code(torch.float32), L.ptr(y), L.ptr(ws), ws.numel(),
                                    L.stream_of(x))
    assert st != 0


@pytest.mark.parametrize("T", [16, 40])
def test_moe_decode_row_pair_down(cuda, T):
    """Routed down projection on pairs of 64-row tiles (chosen once its items fill a wave of
    CTAs: 64 experts x 2048 / 128 pairs here) gives the same bits as single tiles, direct and
    graphed, and matches the oracle."""
    rng = np.random.default_rng(500 + T)
    E, D, I, k = 64, 2048, 256, 6
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    outs = []
    for pair in (True, False):
        for graph in (False, True):
            m = _moe(p, args, round_bf16=False)
            m.row_pair_down, m.cuda_graph = pair, graph
            if not graph:
                L.prof_enable(True)
            y, w, idx = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
            ye = m.experts(_bf(xb), idx)
            if not graph:
                torch.cuda.synchronize()
                names = set(L.prof_report())
                L.prof_enable(False)
                assert ("moe_expert_down_fp4_pairs" in names) == pair
                assert ("moe_expert_down_fp4" in names) == (not pair)
            outs.append((y, w, idx, ye))
    for y, w, idx, ye in outs[1:]:
        assert torch.equal(idx, outs[0][2]) and torch.equal(w, outs[0][1])
        assert torch.equal(y, outs[0][0]) and torch.equal(ye, outs[0][3])
    y, w, idx, _ = outs[0]
    w, idx = w.cpu().numpy(), idx.cpu().numpy()
    want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=False, routing=(w, idx))
    assert rel_fro(y.cpu().numpy(), want) < 1e-5
