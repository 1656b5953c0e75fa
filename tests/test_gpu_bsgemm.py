"""Block-scaled tcgen05 GEMMs and the a8 MoE prefill vs the oracle (upstream numerics).

The a8 oracle quantizes activations with upstream act_quant (bit-exact, checked
first) and multiplies the exactly decoded operands in float64, so the only
difference left is the kernel's fp32 accumulation order:
  * fp32 output: relative Frobenius error < 1e-5;
  * bf16 output: < 1e-2 (bf16 rounding alone is ~2e-3).
The MoE prefill rounds every linear output to bf16 as upstream does and
requantizes h; one-ulp flips of those roundings leave it well inside 1e-2.
"""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import rel_fro
from deepseek_v41_mlx_b200 import _lib as L
from gen import bf16_acts, fp4_weight, fp8_weight, moe_params
from oracle import act_quant as AQ
from oracle import linear as OL
from oracle import moe as OM
from oracle.formats import E4M3, dequant_fp4

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bf(bits):
    return _d(bits.view(np.int16)).view(torch.bfloat16)


def _quant(xb, block):
    a, a_s = q.act_quant.act_quant(_bf(xb), block, "ue8m0", torch.float8_e8m0fnu)
    return a, a_s


def _check_quant(a, a_s, xf, block):
    oq, os_ = AQ.act_quant(xf, block, True)
    assert np.array_equal(L.u8(a).cpu().numpy(), oq)
    assert np.array_equal(L.u8(a_s).cpu().numpy(), AQ.s_to_ue8m0(os_))


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (17, 256, 512), (256, 128, 256),
                                   (300, 384, 1024), (513, 256, 7168)])
def test_fp4_gemm(cuda, M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    xb, xf = bf16_acts(rng, M, K)
    w, s = fp4_weight(rng, N, K)
    a, a_s = _quant(xb, 32)
    _check_quant(a, a_s, xf, 32)
    want = OL.linear_fp4_a8(xf, w, s)
    c32 = q.gemm.fp4_gemm(a, a_s, _d(w), _d(s), act_block_size=32, out_dtype=torch.float32)
    assert rel_fro(c32.cpu().numpy(), want) < 1e-5
    c16 = q.gemm.fp4_gemm(a, a_s, _d(w), _d(s), act_block_size=32, out_dtype=torch.bfloat16)
    assert rel_fro(c16.float().cpu().numpy(), want) < 1e-2


def test_fp4_gemm_act_block_128(cuda):
    rng = np.random.default_rng(5)
    M, N, K = 70, 256, 1024
    xb, xf = bf16_acts(rng, M, K)
    w, s = fp4_weight(rng, N, K)
    a, a_s = _quant(xb, 128)
    _check_quant(a, a_s, xf, 128)
    want = OL._mm(AQ.act_quant_dequant(xf, 128), dequant_fp4(w, s, "f32"))
    c = q.gemm.fp4_gemm(a, a_s, _d(w), _d(s), act_block_size=128, out_dtype=torch.float32)
    assert rel_fro(c.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("M,N,K", [(1, 128, 128), (40, 256, 768), (260, 128, 2048)])
def test_fp8_gemm_block32(cuda, M, N, K):
    rng = np.random.default_rng(M + N * 3 + K)
    xb, xf = bf16_acts(rng, M, K)
    w, s = fp8_weight(rng, N, K)
    a, a_s = _quant(xb, 32)
    want = OL.linear_fp8_block_a8(xf, w, s)
    c = q.gemm.fp8_gemm(a, a_s, _d(w), _d(s), block_size=32, out_dtype=torch.float32)
    assert rel_fro(c.cpu().numpy(), want) < 1e-5
    c16 = q.gemm.fp8_gemm(a, a_s, _d(w), _d(s), block_size=32, out_dtype=torch.bfloat16)
    assert rel_fro(c16.float().cpu().numpy(), want) < 1e-2


def test_fp8_gemm_block128(cuda):
    """Upstream's default 128x128 weight blocks with per-128 activation scales."""
    rng = np.random.default_rng(11)
    M, N, K = 33, 384, 1024
    xb, xf = bf16_acts(rng, M, K)
    w = rng.integers(0, 256, size=(N, K), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0
    s = rng.integers(118, 128, size=(N // 128, K // 128), dtype=np.uint8)
    wd = E4M3[w] * np.repeat(np.repeat(np.exp2(s.astype(np.float64) - 127), 128, 0), 128, 1)
    a, a_s = _quant(xb, 128)
    want = OL._mm(AQ.act_quant_dequant(xf, 128), wd)
    c = q.gemm.fp8_gemm(a, a_s, _d(w), _d(s), block_size=128, out_dtype=torch.float32)
    assert rel_fro(c.cpu().numpy(), want) < 1e-5


def _args(E, D, I, k, limit=10.0):
    return types.SimpleNamespace(n_activated_experts=k, score_func="sqrtsoftplus", gate_temp=1.0,
                                 norm_topk_prob=True, route_scale=1.5, n_routed_experts=E, dim=D,
                                 moe_inter_dim=I, swiglu_limit=limit)


def _moe(p, args):
    m = q.moe.MoE(args, round_bf16=True, cuda_graph=False)
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


# (600, 4, 512, 128, 2) and (900, 4, 384, 256, 2) have wide tiles: the 2-CTA form runs both
# wide launches of the first, and the gate/up one of the second (its down projection has 3
# m-tiles, an odd count, and takes the 1-CTA form)
@pytest.mark.parametrize("T,E,D,I,k", [(5, 8, 256, 128, 3), (70, 8, 256, 256, 3),
                                       (600, 4, 512, 128, 2), (900, 4, 384, 256, 2)])
def test_moe_prefill_given_routing(cuda, T, E, D, I, k):
    rng = np.random.default_rng(T + E + D)
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    w, idx, _ = OM.gate(xf, p["gate_w"], p["gate_bias"], k)
    want, _, _ = OM.moe_forward_upstream_a8(xf, p, _cfg(args), routing=(w, idx))
    m = _moe(p, args)
    y = m.prefill_a8(_bf(xb), weights=_d(w), indices=_d(idx.astype(np.int32)),
                     out_dtype=torch.float32)
    assert rel_fro(y.cpu().numpy(), want) < 1e-2


def test_moe_prefill_router(cuda):
    """Routing computed on the device; the oracle is given the kernel's routing."""
    rng = np.random.default_rng(3)
    T, E, D, I, k = 40, 16, 256, 128, 4
    p = moe_params(rng, E, D, I)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    m = _moe(p, args)
    w, idx = m.gate(_bf(xb))
    y = m.prefill_a8(_bf(xb), out_dtype=torch.float32)
    want, _, _ = OM.moe_forward_upstream_a8(xf, p, _cfg(args),
                                            routing=(w.cpu().numpy(), idx.cpu().numpy()))
    assert rel_fro(y.cpu().numpy(), want) < 1e-2


def test_moe_prefill_no_shared_skewed(cuda):
    """One expert takes most pairs: several full 256-row tiles plus a ragged tail."""
    rng = np.random.default_rng(9)
    T, E, D, I, k = 700, 6, 256, 128, 2
    p = moe_params(rng, E, D, I, with_shared=False)
    args = _args(E, D, I, k)
    xb, xf = bf16_acts(rng, T, D)
    idx = np.stack([np.zeros(T, np.int64), rng.integers(1, E, size=T)], -1)
    w = rng.uniform(0.2, 1.5, size=(T, k)).astype(np.float32)
    want, _, _ = OM.moe_forward_upstream_a8(xf, p, _cfg(args), routing=(w, idx),
                                            with_shared=False)
    m = q.moe.MoE(args, round_bf16=True, cuda_graph=False)
    for name, key in (("gate_proj", "1"), ("up_proj", "3"), ("down_proj", "2")):
        getattr(m.experts, name).weight = _d(p["w" + key])
        getattr(m.experts, name).scales = _d(p["s" + key])
    m.gate.weight = _bf(p["gate_w_bits"])      # shared expert left without weights
    m.gate.bias = _d(p["gate_bias"])
    y = m.prefill_a8(_bf(xb), weights=_d(w), indices=_d(idx.astype(np.int32)),
                     out_dtype=torch.float32)
    assert rel_fro(y.cpu().numpy(), want) < 1e-2
