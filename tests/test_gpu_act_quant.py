"""GPU act_quant vs tests/kernel_stub.py act_quant (golden) and the oracle: bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
from conftest import bits_equal, golden
from oracle import act_quant as AQ

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("i", [0, 1, 2])
def test_act_quant_golden(cuda, i):
    g = golden("act_quant.npz")
    x = torch.from_numpy(g[f"x{i}"]).cuda().to(torch.bfloat16)
    qv, s = q.act_quant.act_quant(x, 32, "ue8m0", torch.float32)
    assert np.array_equal(qv.view(torch.uint8).cpu().numpy(), g[f"codes{i}"])
    assert bits_equal(s.cpu().numpy().reshape(-1), g[f"s{i}"].reshape(-1))
    qf, sf = q.act_quant.act_quant(x, 32, None, torch.float32)
    assert np.array_equal(qf.view(torch.uint8).cpu().numpy(), g[f"codesf{i}"])
    assert bits_equal(sf.cpu().numpy().reshape(-1), g[f"sf{i}"].reshape(-1))
    xi = x.clone()
    q.act_quant.act_quant(xi, 32, "ue8m0", torch.float32, inplace=True)
    assert bits_equal(xi.float().cpu().numpy(), g[f"deq{i}"])


@pytest.mark.parametrize("block", [32, 128])
def test_act_quant_random(cuda, block):
    rng = np.random.default_rng(block)
    x = (rng.standard_normal((65, 1024)) * np.exp(rng.standard_normal((65, 1)) * 3)).astype(np.float32)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    xv = xt.float().cpu().numpy()
    qv, s = q.act_quant.act_quant(xt, block, "ue8m0", torch.float8_e8m0fnu)
    wq, ws = AQ.act_quant(xv, block, True)
    assert np.array_equal(qv.view(torch.uint8).cpu().numpy(), wq)
    assert np.array_equal(s.view(torch.uint8).cpu().numpy(), AQ.s_to_ue8m0(ws))
