"""Weight-decode GEMV kernels vs the oracle's dequant-then-matmul (float64).

Tolerances (relative Frobenius): 1e-5 with fp32 output, 1e-2 with bf16 output.
"""

from __future__ import annotations

import gc

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import rel_fro
from gen import affine_weight, bf16_acts, fp4_weight, fp8_weight
from oracle import formats as F
from oracle import linear as OL

pytestmark = pytest.mark.gpu

TOL_F32, TOL_BF16 = 1e-5, 1e-2


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _x(bits):
    return _d(bits.view(np.int16)).view(torch.bfloat16)


# M = 1 goes to the single-row CUDA-core kernel (k_gemv_fp8_m1): ragged N, K from one 32-code
# block to four passes of a lane's chunk window
@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (5, 200, 256), (8, 64, 128), (16, 130, 384),
                                   (32, 512, 1024), (40, 96, 7168), (1, 4096, 7168),
                                   (1, 70, 32), (1, 33, 16384), (1, 1000, 4160)])
def test_gemv_fp8_block(cuda, M, N, K):
    rng = np.random.default_rng(M * 1000 + N)
    w, s = fp8_weight(rng, N, K)
    xb, xf = bf16_acts(rng, M, K)
    want = OL.linear_fp8_block(xf, w, s)
    got = q.linear.linear_fp8(_x(xb), _d(w), _d(s), out_dtype=torch.float32).cpu().numpy()
    assert rel_fro(got, want) < TOL_F32
    gotb = q.linear.linear_fp8(_x(xb), _d(w), _d(s)).float().cpu().numpy()
    assert rel_fro(gotb, want) < TOL_BF16


@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (3, 70, 256), (16, 64, 2048), (32, 128, 1024),
                                   (33, 64, 512), (8, 2048, 7168)])
def test_gemv_fp4(cuda, M, N, K):
    rng = np.random.default_rng(M * 7 + K)
    w, s = fp4_weight(rng, N, K)
    xb, xf = bf16_acts(rng, M, K)
    want = OL.linear_fp4(xf, w, s)
    got = q.linear.linear_fp4(_x(xb), _d(w), _d(s), out_dtype=torch.float32).cpu().numpy()
    assert rel_fro(got, want) < TOL_F32
    gotb = q.linear.linear_fp4(_x(xb), _d(w), _d(s)).float().cpu().numpy()
    assert rel_fro(gotb, want) < TOL_BF16


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(1, 128, 512), (16, 96, 1024), (7, 64, 256), (32, 64, 512)])
def test_gemv_affine(cuda, bits, M, N, K):
    rng = np.random.default_rng(bits * 100 + M)
    wq, s, b = affine_weight(rng, N, K, bits)
    xb, xf = bf16_acts(rng, M, K)
    want = OL.linear_affine(xf, wq, s, b, bits)
    ts = _d(s.view(np.int16)).view(torch.bfloat16)
    tb = _d(b.view(np.int16)).view(torch.bfloat16)
    got = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)), ts, tb, bits,
                                 out_dtype=torch.float32).cpu().numpy()
    assert rel_fro(got, want) < TOL_F32
    gotb = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)), ts, tb, bits).float().cpu().numpy()
    assert rel_fro(gotb, want) < TOL_BF16


# one activation row: the CUDA-core kernels (k_gemv_affine4_m1, k_gemv_byte_m1<affine>); K from
# one group to two passes of a lane's chunk window, ragged N
@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("N,K", [(14336, 7168), (37, 64), (300, 16384), (1000, 4160)])
def test_gemv_affine_single_row(cuda, bits, N, K):
    rng = np.random.default_rng(N + K + bits)
    wq, s, b = affine_weight(rng, N, K, bits)
    xb, xf = bf16_acts(rng, 1, K)
    ts = _d(s.view(np.int16)).view(torch.bfloat16)
    tb = _d(b.view(np.int16)).view(torch.bfloat16)
    rows = rng.choice(N, min(N, 512), replace=False)
    want = OL.linear_affine(xf, wq[rows], s[rows], b[rows], bits)
    got = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)), ts, tb, bits,
                                 out_dtype=torch.float32)
    assert rel_fro(got.cpu().numpy()[:, rows], want) < TOL_F32
    again = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)), ts, tb, bits,
                                   out_dtype=torch.float32)
    assert torch.equal(got, again)                         # fixed summation order
    gotb = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)), ts, tb, bits).float().cpu().numpy()
    assert rel_fro(gotb[:, rows], want) < TOL_BF16


def test_gemv_affine_baseline_shape(cuda):
    """config 4 weight [14336, 7168] 4-bit, M = 16, against the oracle on a row sample."""
    rng = np.random.default_rng(4)
    N, K, M = 14336, 7168, 16
    wq, s, b = affine_weight(rng, N, K, 4)
    xb, xf = bf16_acts(rng, M, K)
    ts = _d(s.view(np.int16)).view(torch.bfloat16)
    tb = _d(b.view(np.int16)).view(torch.bfloat16)
    got = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)), ts, tb, 4,
                                 out_dtype=torch.float32).cpu().numpy()
    rows = rng.choice(N, 256, replace=False)
    want = OL.linear_affine(xf, wq[rows], s[rows], b[rows], 4)
    assert rel_fro(got[:, rows], want) < TOL_F32


def test_gemv_repeat_is_deterministic(cuda):
    """split-K partial sums are reduced in a fixed order: identical bits on repeat."""
    rng = np.random.default_rng(9)
    w, s = fp8_weight(rng, 4096, 7168)
    xb, _ = bf16_acts(rng, 1, 7168)
    a = q.linear.linear_fp8(_x(xb), _d(w), _d(s), out_dtype=torch.float32)
    b = q.linear.linear_fp8(_x(xb), _d(w), _d(s), out_dtype=torch.float32)
    assert torch.equal(a, b)


def test_gemv_extreme_scales_exact(cuda):
    """ue8m0 scales over the whole exponent range stay exact (scale folded in fp32)."""
    rng = np.random.default_rng(11)
    N, K = 64, 256
    w, _ = fp4_weight(rng, N, K)
    s = rng.integers(1, 200, size=(N, K // 32), dtype=np.uint8)
    xb, xf = bf16_acts(rng, 2, K)
    want = OL.linear_fp4(xf, w, s)
    got = q.linear.linear_fp4(_x(xb), _d(w), _d(s), out_dtype=torch.float32).cpu().numpy()
    assert rel_fro(got, want) < TOL_F32


def test_gemv_large_activations(cuda):
    """per-row power-of-two activation scaling keeps huge / tiny rows exact."""
    rng = np.random.default_rng(12)
    N, K = 128, 512
    w, s = fp8_weight(rng, N, K)
    xb, xf = bf16_acts(rng, 3, K)
    xf = xf * np.array([[1e30], [1e-30], [1.0]], dtype=np.float32)
    xb = F.f32_to_bf16_bits(xf)
    xf = F.bf16_bits_to_f32(xb)
    want = OL.linear_fp8_block(xf, w, s)
    got = q.linear.linear_fp8(_x(xb), _d(w), _d(s), out_dtype=torch.float32).cpu().numpy()
    for r in range(3):
        assert rel_fro(got[r], want[r]) < TOL_F32


@pytest.mark.parametrize("bits", [0, 4, 8])
def test_gemv_single_row_large_activations(cuda, bits):
    """The single-row kernels (fp8: per-row power-of-two f16 copy of x; affine: bf16 / f16 x)
    on huge and tiny activation rows: each row alone against the oracle."""
    rng = np.random.default_rng(13 + bits)
    N, K = 96, 1024
    for mult in (1e30, 1e-30, 1.0):
        xb, xf = bf16_acts(rng, 1, K)
        xb = F.f32_to_bf16_bits(xf * np.float32(mult))
        xf = F.bf16_bits_to_f32(xb)
        if bits == 0:
            w, sc = fp8_weight(rng, N, K)
            want = OL.linear_fp8_block(xf, w, sc)
            got = q.linear.linear_fp8(_x(xb), _d(w), _d(sc), out_dtype=torch.float32)
        else:
            wq, sa, ba = affine_weight(rng, N, K, bits)
            want = OL.linear_affine(xf, wq, sa, ba, bits)
            got = q.linear.linear_affine(_x(xb), _d(wq.view(np.int32)),
                                         _d(sa.view(np.int16)).view(torch.bfloat16),
                                         _d(ba.view(np.int16)).view(torch.bfloat16), bits,
                                         out_dtype=torch.float32)
        assert rel_fro(got.cpu().numpy(), want) < TOL_F32, mult


def test_gemv_fp8_single_row_matches_engine_on_edge_codes(cuda):
    """NaN codes, scale bytes 0 (applied as 0) to 200: the single-row kernel and the
    tensor-core engine (a two-row call) give the same NaN pattern and agree elsewhere."""
    rng = np.random.default_rng(14)
    N, K = 160, 2048
    w = rng.integers(0, 256, size=(N, K), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0
    w[5, 100] = 0x7F                                     # NaN codes in rows 5 and 77
    w[77, 2000] = 0xFF
    s = rng.integers(0, 201, size=((N + 31) // 32, K // 32), dtype=np.uint8)
    s[0, 0] = 0
    xb, _ = bf16_acts(rng, 2, K)
    one = q.linear.linear_fp8(_x(xb[:1]), _d(w), _d(s), out_dtype=torch.float32).cpu().numpy()
    two = q.linear.linear_fp8(_x(xb), _d(w), _d(s), out_dtype=torch.float32).cpu().numpy()[:1]
    assert np.array_equal(np.isnan(one), np.isnan(two))
    assert np.isnan(one[0, 5]) and np.isnan(one[0, 77])
    fin = ~np.isnan(one) & np.isfinite(two)
    assert rel_fro(one[fin], two[fin]) < TOL_F32


@pytest.mark.parametrize("M", [1, 32])
def test_gemv_chain_in_graph_matches_eager(cuda, M):
    """Consecutive dense GEMVs replayed from one CUDA graph -- each one launched as the
    programmatic dependent of its activation prep, issuing weight copies before that kernel
    has finished, with the split-K tickets zeroed by the prep -- give the bits of the same
    calls made one at a time, and the oracle's values."""
    rng = np.random.default_rng(41 + M)
    N, K, n = 4096, 7168, 3
    ws = [fp8_weight(rng, N, K) for _ in range(n)]
    xs = [bf16_acts(rng, M, K) for _ in range(n)]
    tw = [(_d(w), _d(s)) for w, s in ws]
    tx = [_x(xb) for xb, _ in xs]
    eager = [q.linear.linear_fp8(tx[i], *tw[i], out_dtype=torch.float32) for i in range(n)]
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        [q.linear.linear_fp8(tx[i], *tw[i], out_dtype=torch.float32) for i in range(n)]
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    gc.collect()                  # no finalizer of an earlier test's CUDA objects mid-capture
    gc.disable()
    try:
        with torch.cuda.graph(g):
            outs = [q.linear.linear_fp8(tx[i], *tw[i], out_dtype=torch.float32) for i in range(n)]
    finally:
        gc.enable()
    for _ in range(2):
        for o in outs:
            o.zero_()
        g.replay()
        torch.cuda.synchronize()
        for i in range(n):
            assert torch.equal(outs[i], eager[i]), i
    want = OL.linear_fp8_block(xs[0][1], ws[0][0], ws[0][1])
    assert rel_fro(outs[0].cpu().numpy(), want) < TOL_F32
