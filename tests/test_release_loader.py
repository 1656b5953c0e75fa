"""The release-checkpoint loader on CPU: config mapping, raw bytes of every tensor, and the
per-rank selection of experts and engram rows (no compute)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import deepseek_v41_mlx_b200 as q
import release_fixture as RF


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    path, arrays = RF.write(str(tmp_path_factory.mktemp("release")))
    return q.release.Checkpoint(path), arrays


def test_config_mapping(ckpt):
    c, _ = ckpt
    a = c.args
    assert (a.dim, a.moe_inter_dim, a.n_routed_experts, a.n_activated_experts) == \
        (RF.D, RF.I, RF.E, RF.K)
    assert a.score_func == "sqrtsoftplus" and a.route_scale == 1.5 and a.swiglu_limit == 10.0
    assert a.engram_layer_ids == (RF.ENGRAM_LAYER,) and a.engram_head_dim == RF.HD


def test_moe_tensors_are_the_release_bytes(ckpt):
    c, arr = ckpt
    p = arr["moe"]
    m = q.release.load_moe(c, RF.MOE_LAYER, device="cpu")
    assert m.gate.weight.dtype == torch.bfloat16
    assert np.array_equal(m.gate.weight.view(torch.int16).numpy(), p["gate_w_bits"].view(np.int16))
    assert np.array_equal(m.gate.bias.numpy(), p["gate_bias"])
    for wn, proj in (("w1", "gate_proj"), ("w3", "up_proj"), ("w2", "down_proj")):
        pr = getattr(m.experts, proj)
        assert pr.weight.dtype == torch.uint8 and np.array_equal(pr.weight.numpy(), p[wn])
        assert np.array_equal(pr.scales.numpy(), p["s" + wn[1]])
    for wn in ("w1", "w2", "w3"):
        pr = getattr(m.shared_experts, wn)
        assert np.array_equal(pr.weight.numpy(), p["s" + wn])
        assert np.array_equal(pr.scales.numpy(), p["ss" + wn[1]])


def test_moe_rank_reads_only_its_experts(ckpt):
    c, arr = ckpt
    p = arr["moe"]
    world = 2
    for rank in range(world):
        e = q.release.load_moe(c, RF.MOE_LAYER, device="cpu", rank=rank, world=world)
        epr = RF.E // world
        assert e.epr == epr and e.topk == RF.K
        w1 = e.local.experts.gate_proj.weight.numpy()
        assert w1.shape[0] == epr
        assert np.array_equal(w1, p["w1"][rank * epr:(rank + 1) * epr])
        assert e.gate_w.shape[0] == RF.E                  # the router covers every expert


def test_engram_tables_and_row_shards(ckpt):
    c, arr = ckpt
    g = q.release.load_engram(c, RF.ENGRAM_LAYER, device="cpu")
    assert np.array_equal(g.embed.weight.numpy(), arr["table"])
    assert np.array_equal(g.embed.scale.numpy(), arr["tscale"])
    assert g.embed.block == 32
    assert np.array_equal(g.wkv.weight.numpy(), arr["wkv"])
    assert np.array_equal(g.q_weight.numpy(), arr["q_weight"])
    for rank in range(3):
        gs = q.release.load_engram(c, RF.ENGRAM_LAYER, device="cpu", rank=rank, world=3)
        part = -(-RF.ROWS // 3)
        lo, hi = rank * part, min(RF.ROWS, (rank + 1) * part)
        assert gs.embed.part == part and gs.embed.row_lo == lo
        assert np.array_equal(gs.embed.weight.numpy(), arr["table"][lo:hi])


def test_shapes_from_headers(ckpt):
    c, _ = ckpt
    assert c.shape(f"layers.{RF.ENGRAM_LAYER}.engram.embed.weight") == (RF.ROWS, RF.HD)
    assert c.shape(f"layers.{RF.ENGRAM_LAYER}.engram.embed.scale") == (RF.ROWS, RF.HD // 32)
    assert c.shape(f"layers.{RF.MOE_LAYER}.ffn.experts.0.w1.weight") == (RF.I, RF.D // 2)
    with pytest.raises(KeyError):
        c.shape("no.such.weight")
