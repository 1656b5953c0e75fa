"""MLX affine quantized matmul at prefill sizes (tcgen05 kind::f16) vs the oracle.

The tensor-core path multiplies weights dequantized to bf16 (round(fma_f32(s, q, b)), the
mx.dequantize values) with the bf16 activations: against the oracle of exactly that
definition (float64 accumulation) the fp32 output agrees to 1e-5 relative Frobenius; against
the exact-affine oracle (no weight rounding) the bf16 weight rounding stays under 1e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import rel_fro
from gen import affine_weight, bf16_acts
from oracle import linear as OL

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bf(bits):
    return _d(bits.view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K", [(65, 128, 64), (300, 256, 512), (513, 384, 1024)])
def test_qmm_affine(cuda, bits, M, N, K):
    rng = np.random.default_rng(bits * 1000 + M + N)
    wq, s, b = affine_weight(rng, N, K, bits)
    xb, xf = bf16_acts(rng, M, K)
    want = OL.linear_affine_bf16w(xf, wq, s, b, bits)
    args = (_bf(xb), _d(wq.view(np.int32)), _bf(s), _bf(b), bits)
    got = q.linear.linear_affine(*args, out_dtype=torch.float32).cpu().numpy()
    assert rel_fro(got, want) < 1e-5
    assert rel_fro(got, OL.linear_affine(xf, wq, s, b, bits)) < 1e-2
    got16 = q.linear.linear_affine(*args).float().cpu().numpy()
    assert rel_fro(got16, want) < 1e-2


def test_qmm_affine_baseline_shape(cuda):
    """BASELINE configs[3] at prefill: [14336, 7168] 4-bit, M = 4096, a row sample checked."""
    rng = np.random.default_rng(44)
    N, K, M = 14336, 7168, 4096
    wq, s, b = affine_weight(rng, N, K, 4)
    xb, xf = bf16_acts(rng, M, K)
    got = q.linear.linear_affine(_bf(xb), _d(wq.view(np.int32)), _bf(s), _bf(b), 4,
                                 out_dtype=torch.float32).cpu().numpy()
    rows = rng.choice(N, 128, replace=False)
    toks = rng.choice(M, 256, replace=False)
    want = OL.linear_affine_bf16w(xf[toks], wq[rows], s[rows], b[rows], 4)
    assert rel_fro(got[np.ix_(toks, rows)], want) < 1e-5
