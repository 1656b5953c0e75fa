"""Modules loaded from a release-layout checkpoint compute exactly what the same modules
built from the arrays compute (MoE decode and prefill, engram lookup + gate)."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
import release_fixture as RF
from gen import bf16_acts

pytestmark = pytest.mark.gpu


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    path, arrays = RF.write(str(tmp_path_factory.mktemp("release_gpu")))
    return q.release.Checkpoint(path), arrays


def test_loaded_moe_matches_direct(cuda, ckpt):
    c, arr = ckpt
    p = arr["moe"]
    m = q.release.load_moe(c, RF.MOE_LAYER, device="cuda")
    ref = q.moe.MoE(c.args)
    ref.gate.weight = _d(p["gate_w_bits"].view(np.int16)).view(torch.bfloat16)
    ref.gate.bias = _d(p["gate_bias"])
    for wn, proj in (("w1", "gate_proj"), ("w3", "up_proj"), ("w2", "down_proj")):
        getattr(ref.experts, proj).weight = _d(p[wn])
        getattr(ref.experts, proj).scales = _d(p["s" + wn[1]])
    for wn in ("w1", "w2", "w3"):
        getattr(ref.shared_experts, wn).weight = _d(p["s" + wn])
        getattr(ref.shared_experts, wn).scales = _d(p["ss" + wn[1]])
    rng = np.random.default_rng(4)
    for T in (1, 9):
        xb, _ = bf16_acts(rng, T, RF.D)
        x = _d(xb.view(np.int16)).view(torch.bfloat16)
        assert torch.equal(m(x), ref(x))
        assert torch.equal(m.prefill_a8(x), ref.prefill_a8(x))


def test_loaded_engram_matches_direct(cuda, ckpt):
    c, arr = ckpt
    g = q.release.load_engram(c, RF.ENGRAM_LAYER, device="cuda")
    ref = q.engram.Engram(c.args, 0)
    ref.embed.weight, ref.embed.scale = _d(arr["table"]), _d(arr["tscale"])
    ref.wkv = q.linear.FP8Linear(_d(arr["wkv"]), _d(arr["wkv_s"]))
    ref.q_weight, ref.k_weight = _d(arr["q_weight"]), _d(arr["k_weight"])
    rng = np.random.default_rng(6)
    B, Lq = 2, 5
    xb, _ = bf16_acts(rng, B * Lq * RF.HC, RF.D)
    x = _d(xb.view(np.int16)).view(torch.bfloat16).reshape(B, Lq, RF.HC, RF.D)
    ids = _d(rng.integers(0, RF.ROWS, size=(B, Lq, 3 * RF.HEADS)))
    assert torch.equal(g(x, ids), ref(x, ids))
