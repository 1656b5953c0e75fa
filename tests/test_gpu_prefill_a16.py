"""The MoE layer at prefill sizes in the port's numerics on the tensor cores
(``MoE.prefill_a16``, ``dsv41_moe_prefill_a16``) against the oracle's port of
deepseek_v41_mlx/moe.py:96-112 (``oracle.moe.moe_forward``): 1e-5 relative Frobenius with
every intermediate in fp32 (exact mode, fp32 output) and 1e-2 with the port's bf16
rounding (bf16 output).  The routed down projection takes the fp32 SwiGLU output as bf16
hi + lo halves, which leaves ~2^-18 per element."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import rel_fro
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


def _cfg(args):
    return dict(topk=args.n_activated_experts, score_func="sqrtsoftplus", gate_temp=1.0,
                norm_topk_prob=True, route_scale=1.5, swiglu_limit=args.swiglu_limit)


def _moe(p, args, round_bf16, with_shared=True):
    m = q.moe.MoE(args, round_bf16=round_bf16, cuda_graph=False)
    m.gate.weight = _bf(p["gate_w_bits"])
    m.gate.bias = _d(p["gate_bias"])
    for name, key in (("gate_proj", "1"), ("up_proj", "3"), ("down_proj", "2")):
        getattr(m.experts, name).weight = _d(p["w" + key])
        getattr(m.experts, name).scales = _d(p["s" + key])
    if with_shared:
        for key in ("1", "2", "3"):
            getattr(m.shared_experts, "w" + key).weight = _d(p["sw" + key])
            getattr(m.shared_experts, "w" + key).scales = _d(p["ss" + key])
    return m


@pytest.mark.parametrize("T,E,D,I,k", [(5, 8, 256, 128, 3), (70, 8, 256, 256, 3),
                                       (600, 4, 512, 128, 2), (300, 16, 384, 256, 6)])
def test_prefill_a16_given_routing(cuda, T, E, D, I, k):
    rng = np.random.default_rng(T + E + D + I)
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    w, idx, _ = OM.gate(xf, p["gate_w"], p["gate_bias"], k)
    for exact in (True, False):
        m = _moe(p, args, round_bf16=not exact)
        y = m.prefill_a16(_bf(xb), weights=_d(w), indices=_d(idx.astype(np.int32)),
                          out_dtype=torch.float32 if exact else torch.bfloat16)
        want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=not exact, routing=(w, idx))
        assert rel_fro(y.float().cpu().numpy(), want) < (1e-5 if exact else 1e-2), exact


def test_prefill_a16_router(cuda):
    """Routing computed on the device; the oracle is given the kernel's routing."""
    rng = np.random.default_rng(3)
    T, E, D, I, k = 40, 16, 256, 128, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    m = _moe(p, args, round_bf16=False)
    w, idx = m.gate(_bf(xb))
    y = m.prefill_a16(_bf(xb), out_dtype=torch.float32)
    want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=False,
                                routing=(w.cpu().numpy(), idx.cpu().numpy()))
    assert rel_fro(y.cpu().numpy(), want) < 1e-5


def test_prefill_a16_skewed_no_shared(cuda):
    """One expert takes most pairs: several full 224-row tiles plus a ragged tail; no shared
    expert; and the shared expert alone (routed=False)."""
    rng = np.random.default_rng(9)
    T, E, D, I, k = 700, 6, 256, 128, 2
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    idx = np.stack([np.zeros(T, np.int64), rng.integers(1, E, size=T)], -1)
    w = rng.uniform(0.2, 1.5, size=(T, k)).astype(np.float32)
    m = _moe(p, args, round_bf16=False)
    y = m.prefill_a16(_bf(xb), weights=_d(w), indices=_d(idx.astype(np.int32)),
                      out_dtype=torch.float32, shared=False)
    want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=False, with_shared=False,
                                routing=(w, idx))
    assert rel_fro(y.cpu().numpy(), want) < 1e-5
    ys = m.prefill_a16(_bf(xb), out_dtype=torch.float32, routed=False)
    sh = OM.shared_expert_fp8(xf, p["sw1"], p["ss1"], p["sw3"], p["ss3"], p["sw2"], p["ss2"],
                              10.0, False)
    assert rel_fro(ys.cpu().numpy(), sh) < 1e-5


def test_prefill_a16_matches_decode_path(cuda):
    """The tensor-core prefill and the decode engine compute the same port numerics: their
    outputs agree at 1e-5 (exact mode, fp32), on the same routing."""
    rng = np.random.default_rng(21)
    T, E, D, I, k = 96, 12, 512, 256, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, _ = bf16_acts(rng, T, D)
    m = _moe(p, args, round_bf16=False)
    y_dec, w, idx = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
    y_pf = m.prefill_a16(_bf(xb), weights=w, indices=idx, out_dtype=torch.float32)
    assert rel_fro(y_pf.cpu().numpy(), y_dec.cpu().numpy()) < 1e-5


def test_prefill_a16_scale_byte_edges(cuda):
    """Scale bytes far from 127: down-projection scale bytes drawn from 8..16 (weights near
    2^-115, the outputs near 2^-110, still normal fp32; the error bound is relative) decode
    exactly like the release's scales."""
    rng = np.random.default_rng(33)
    T, E, D, I, k = 150, 8, 256, 256, 3
    p = moe_params(rng, E, D, I)
    p["s2"] = rng.integers(8, 17, size=p["s2"].shape, dtype=np.uint8)
    p["s1"] = rng.integers(15, 17, size=p["s1"].shape, dtype=np.uint8) + np.uint8(105)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    w, idx, _ = OM.gate(xf, p["gate_w"], p["gate_bias"], k)
    m = _moe(p, args, round_bf16=False)
    y = m.prefill_a16(_bf(xb), weights=_d(w), indices=_d(idx.astype(np.int32)),
                      out_dtype=torch.float32, shared=False)
    want, _, _ = OM.moe_forward(xf, p, _cfg(args), round_bf16_io=False, with_shared=False,
                                routing=(w, idx))
    assert np.abs(want).max() > 0 and np.isfinite(y.cpu().numpy()).all()
    assert rel_fro(y.cpu().numpy(), want) < 1e-5


def test_moe_call_above_crossover_runs_a16(cuda):
    """``MoE.__call__`` above ``a16_min_tokens`` tokens runs the tensor-core path: the same
    routing and the decode engine's outputs within 1e-5 (exact mode, fp32)."""
    rng = np.random.default_rng(23)
    T, E, D, I, k = 40, 12, 256, 128, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, _ = bf16_acts(rng, T, D)
    m = _moe(p, args, round_bf16=False)
    y_dec, w_dec, i_dec = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
    m.a16_min_tokens = 16
    y_a16, w_a16, i_a16 = m(_bf(xb), with_routing=True, out_dtype=torch.float32)
    assert torch.equal(i_dec, i_a16) and torch.equal(w_dec, w_a16)
    assert rel_fro(y_a16.cpu().numpy(), y_dec.cpu().numpy()) < 1e-5
