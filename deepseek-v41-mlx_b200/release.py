"""The native release checkpoint loaded straight into this package's modules.

The hub's safetensors shards keep the quantized formats the kernels read, so nothing is
converted: fp8 e4m3 weights with ue8m0 scales per 32x32 block, fp4 e2m1 expert weights two
per byte (int8 ``[out, in/2]``) with ue8m0 ``[out, in/32]`` scales, engram tables as fp8 rows
with ue8m0 row scales (docs/upstream-notes.md:170-195; tensor names as the reference's
converter reads them, deepseek_v41_mlx/convert.py:91-153, where every such tensor is
dequantized to bf16 first).  Tensors are read as raw bytes and moved to the device as they
are.  An expert-parallel rank reads only its own experts, a row-sharded engram rank only its
own rows (safetensors slices), so no rank ever holds the whole layer.

    ckpt = Checkpoint("/path/to/release")           # config.json + *.safetensors
    args = ckpt.args
    moe = load_moe(ckpt, layer=3, device="cuda")     # moe.MoE (or ep.EPMoE with world > 1)
    eng = load_engram(ckpt, layer_id=1, device="cuda")
"""

from __future__ import annotations

import glob
import json
import os
import types

from . import _lib as L


def _get(c, *names, default=None):
    for n in names:
        if n in c:
            return c[n]
    return default


def args_from_config(cfg):
    """The fields of the hub config (``config.json``, ``text_config`` folded over the top
    level) that the MoE / engram modules use, under the reference's ModelArgs names
    (deepseek_v41_mlx/config.py:136-197)."""
    if isinstance(cfg, str):
        with open(cfg) as f:
            cfg = json.load(f)
    c = dict(cfg)
    if "text_config" in c:
        tc = c.pop("text_config")
        c = {**c, **tc}
    return types.SimpleNamespace(
        dim=_get(c, "hidden_size", "dim", default=5120),
        moe_inter_dim=_get(c, "moe_intermediate_size", "moe_inter_dim", default=2304),
        n_routed_experts=_get(c, "n_routed_experts", default=384),
        n_shared_experts=_get(c, "n_shared_experts", default=1),
        n_activated_experts=_get(c, "num_experts_per_tok", "n_activated_experts", default=6),
        score_func=_get(c, "scoring_func", "score_func", default="sqrtsoftplus"),
        gate_temp=_get(c, "gate_temp", default=1.0),
        norm_topk_prob=_get(c, "norm_topk_prob", default=True),
        route_scale=_get(c, "routed_scaling_factor", "route_scale", default=1.5),
        swiglu_limit=_get(c, "swiglu_limit", default=0.0),
        norm_eps=_get(c, "rms_norm_eps", "norm_eps", default=1e-20),
        hc_mult=_get(c, "hc_mult", default=4),
        engram_layer_ids=tuple(_get(c, "engram_layer_ids", default=()) or ()),
        engram_num_embeddings=tuple(_get(c, "engram_num_embeddings", default=()) or ()),
        engram_max_ngram_size=_get(c, "engram_max_ngram_size", default=4),
        engram_vocab_size=_get(c, "engram_vocab_size", default=0),
        engram_n_heads=_get(c, "engram_n_heads", default=0),
        engram_head_dim=_get(c, "engram_head_dim", default=0),
        engram_pad_id=_get(c, "engram_pad_token_id", "engram_pad_id", default=2),
        engram_compressed_vocab_size=_get(c, "engram_compressed_vocab_size", default=0),
    )


class Checkpoint:
    """Index of a release directory: every tensor name -> its shard."""

    def __init__(self, path: str):
        from safetensors import safe_open
        self.path = path
        self._open = safe_open
        cfg = os.path.join(path, "config.json")
        self.args = args_from_config(cfg) if os.path.exists(cfg) else None
        self.where = {}
        files = sorted(glob.glob(os.path.join(path, "*.safetensors")))
        if not files:
            raise ValueError(f"no *.safetensors in {path}")
        for fn in files:
            with safe_open(fn, framework="pt") as f:
                for k in f.keys():
                    self.where[k] = fn

    def __contains__(self, key):
        return key in self.where

    def shape(self, key):
        """The stored shape of tensor ``key`` (read from the shard header, no data)."""
        if key not in self.where:
            raise KeyError(f"{key} is not in the checkpoint")
        with self._open(self.where[key], framework="pt") as f:
            return tuple(f.get_slice(key).get_shape())

    def get(self, key, device="cuda", rows=None):
        """The tensor ``key`` (rows [lo, hi) of it with ``rows=(lo, hi)``) on ``device``; fp8,
        ue8m0 and int8 tensors come back as their bytes (uint8), others as stored."""
        t = L.torch()
        if key not in self.where:
            raise KeyError(f"{key} is not in the checkpoint")
        with self._open(self.where[key], framework="pt") as f:
            if rows is None:
                v = f.get_tensor(key)
            else:
                v = f.get_slice(key)[rows[0]:rows[1]]
        if v.dtype in (t.float8_e4m3fn, t.float8_e8m0fnu, t.int8):
            v = v.view(t.uint8)
        return v.contiguous().to(device)


def _stack_experts(ckpt, prefix, lo, hi, wn, device):
    t = L.torch()
    ws = [ckpt.get(f"{prefix}.experts.{e}.{wn}.weight", "cpu") for e in range(lo, hi)]
    ss = [ckpt.get(f"{prefix}.experts.{e}.{wn}.scale", "cpu") for e in range(lo, hi)]
    return t.stack(ws).to(device), t.stack(ss).to(device)


def load_moe(ckpt, layer: int, args=None, device="cuda", rank: int = 0, world: int = 1,
             group=None, **moe_kwargs):
    """``layers.{layer}.ffn`` -> ``moe.MoE`` with the router, the shared expert and the
    experts (all of them for world = 1; experts [rank*E/world, (rank+1)*E/world) renumbered
    from 0 inside an ``ep.EPMoE`` otherwise)."""
    from . import ep as EP
    from . import moe as M
    t = L.torch()
    args = args or ckpt.args
    prefix = f"layers.{layer}.ffn"
    E = args.n_routed_experts
    if E % world:
        raise ValueError(f"{E} experts do not split over {world} ranks")
    epr = E // world
    lo, hi = rank * epr, (rank + 1) * epr
    la = types.SimpleNamespace(**vars(args))
    la.n_routed_experts = epr
    m = M.MoE(la, **moe_kwargs)
    gate_w = ckpt.get(f"{prefix}.gate.weight", device).to(t.bfloat16)
    gate_b = ckpt.get(f"{prefix}.gate.bias", device).float() if f"{prefix}.gate.bias" in ckpt \
        else None
    m.gate.weight, m.gate.bias = gate_w, gate_b
    for wn, proj in (("w1", "gate_proj"), ("w3", "up_proj"), ("w2", "down_proj")):
        w, s = _stack_experts(ckpt, prefix, lo, hi, wn, device)
        getattr(m.experts, proj).weight = w
        getattr(m.experts, proj).scales = s
    if args.n_shared_experts:
        for wn in ("w1", "w2", "w3"):
            pr = getattr(m.shared_experts, wn)
            pr.weight = ckpt.get(f"{prefix}.shared_experts.{wn}.weight", device)
            pr.scales = ckpt.get(f"{prefix}.shared_experts.{wn}.scale", device)
    if world == 1:
        return m
    e = EP.EPMoE(m, world, rank, E, group=group)
    e.gate_w, e.gate_b = gate_w, gate_b if gate_b is not None else \
        t.zeros(E, dtype=t.float32, device=gate_w.device)
    e.topk = args.n_activated_experts
    return e


def _packed_table(ckpt, prefix, rows, hd, block, device, chunk=1 << 20):
    """The table read in row chunks and stored packed (codes then scales a row) on the device:
    the unpacked table is never whole on the device."""
    t = L.torch()
    rb = int(L.load().dsv41_engram_row_bytes(hd, block))
    out = t.empty((rows, rb), dtype=t.uint8, device=device)
    for r0 in range(0, rows, chunk):
        r1 = min(rows, r0 + chunk)
        w = ckpt.get(f"{prefix}.embed.weight", device, rows=(r0, r1))
        s = ckpt.get(f"{prefix}.embed.scale", device, rows=(r0, r1))
        L.call("dsv41_engram_pack_rows", L.ptr(w), L.ptr(s), r1 - r0, 0, hd, block, None, r1 - r0,
               L.ptr(out) + r0 * rb, L.stream_of(w))
    return out


def load_engram(ckpt, layer_id: int, args=None, device="cuda", rank: int = 0, world: int = 1,
                group=None, packed: bool = True):
    """``layers.{layer_id}.engram`` -> ``engram.Engram``: the fp8 row table (this rank's rows
    only when world > 1, as a ``ParallelEngramEmbedding``), the fp8 ``wkv`` projection and the
    gate weights.  ``packed`` (one GPU): the table is stored as packed rows (see
    ``EngramEmbedding.pack``), built chunk by chunk while reading."""
    from . import engram as G
    from .linear import FP8Linear
    t = L.torch()
    args = args or ckpt.args
    idx = args.engram_layer_ids.index(layer_id)
    prefix = f"layers.{layer_id}.engram"
    g = G.Engram(args, idx)
    rows = args.engram_num_embeddings[idx]
    hd = args.engram_head_dim
    block = hd // ckpt.get(f"{prefix}.embed.scale", "cpu", rows=(0, 1)).shape[-1]
    if world == 1:
        emb = G.EngramEmbedding(rows, hd, block)
        if packed and str(device).startswith("cuda"):
            emb.packed = _packed_table(ckpt, prefix, rows, hd, block, device)
        else:
            emb.weight = ckpt.get(f"{prefix}.embed.weight", device)
            emb.scale = ckpt.get(f"{prefix}.embed.scale", device)
    else:
        emb = G.ParallelEngramEmbedding(rows, hd, block, rank=rank, world=world, group=group)
        r0 = min(rows, rank * emb.part)
        r1 = min(rows, r0 + emb.part)
        emb.weight = ckpt.get(f"{prefix}.embed.weight", device, rows=(r0, r1))
        emb.scale = ckpt.get(f"{prefix}.embed.scale", device, rows=(r0, r1))
    g.embed = emb
    g.wkv = FP8Linear(ckpt.get(f"{prefix}.wkv.weight", device),
                      ckpt.get(f"{prefix}.wkv.scale", device))
    for name in ("q_weight", "k_weight"):
        key = f"{prefix}.{name}"
        if key in ckpt:
            setattr(g, name, ckpt.get(key, device).float())
    return g
