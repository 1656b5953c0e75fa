"""A tiny synthetic checkpoint in the release's layout (hub config + safetensors shards with
the release dtypes: int8 fp4 experts, F8_E4M3 fp8 weights, F8_E8M0 scales, bf16 router,
fp32 bias), shared by the CPU and GPU loader tests."""

from __future__ import annotations

import json
import os

import numpy as np
import torch

from gen import fp8_weight, moe_params

E, D, I, K = 8, 256, 256, 2
ROWS, HD, HEADS, HC = 1000, 256, 2, 4
MOE_LAYER, ENGRAM_LAYER = 0, 1


def write(dirname, seed=3):
    """-> (path, arrays): the checkpoint directory and the numpy arrays written to it."""
    from safetensors.torch import save_file
    rng = np.random.default_rng(seed)
    p = moe_params(rng, E, D, I)
    cols = 3 * HEADS
    a = {"moe": p}
    a["table"] = rng.integers(0, 126, size=(ROWS, HD), dtype=np.uint8)
    a["tscale"] = rng.integers(115, 124, size=(ROWS, HD // 32), dtype=np.uint8)
    a["wkv"], a["wkv_s"] = fp8_weight(rng, (HC + 1) * D, cols * HD, 112, 120)
    a["q_weight"] = (1.0 + 0.1 * rng.standard_normal((HC, D))).astype(np.float32)
    a["k_weight"] = (1.0 + 0.1 * rng.standard_normal((HC, D))).astype(np.float32)

    def u8(x, dt):
        return torch.from_numpy(np.ascontiguousarray(x)).view(dt).clone()

    f8, e8 = torch.float8_e4m3fn, torch.float8_e8m0fnu
    s1 = {}
    pre = f"layers.{MOE_LAYER}.ffn"
    s1[f"{pre}.gate.weight"] = torch.from_numpy(p["gate_w_bits"].view(np.int16)).view(torch.bfloat16).clone()
    s1[f"{pre}.gate.bias"] = torch.from_numpy(p["gate_bias"]).clone()
    for e in range(E):
        for wn in ("w1", "w3", "w2"):
            s1[f"{pre}.experts.{e}.{wn}.weight"] = u8(p[wn][e], torch.int8)
            s1[f"{pre}.experts.{e}.{wn}.scale"] = u8(p["s" + wn[1]][e], e8)
    for wn in ("w1", "w2", "w3"):
        s1[f"{pre}.shared_experts.{wn}.weight"] = u8(p["s" + wn], f8)
        s1[f"{pre}.shared_experts.{wn}.scale"] = u8(p["ss" + wn[1]], e8)
    s2 = {}
    pre = f"layers.{ENGRAM_LAYER}.engram"
    s2[f"{pre}.embed.weight"] = u8(a["table"], f8)
    s2[f"{pre}.embed.scale"] = u8(a["tscale"], e8)
    s2[f"{pre}.wkv.weight"] = u8(a["wkv"], f8)
    s2[f"{pre}.wkv.scale"] = u8(a["wkv_s"], e8)
    s2[f"{pre}.q_weight"] = torch.from_numpy(a["q_weight"]).to(torch.bfloat16)
    s2[f"{pre}.k_weight"] = torch.from_numpy(a["k_weight"]).to(torch.bfloat16)
    a["q_weight"] = s2[f"{pre}.q_weight"].float().numpy()
    a["k_weight"] = s2[f"{pre}.k_weight"].float().numpy()
    os.makedirs(dirname, exist_ok=True)
    save_file(s1, os.path.join(dirname, "model-00001-of-00002.safetensors"))
    save_file(s2, os.path.join(dirname, "model-00002-of-00002.safetensors"))
    cfg = {"architectures": ["DeepseekV41"], "text_config": {
        "hidden_size": D, "moe_intermediate_size": I, "n_routed_experts": E,
        "num_experts_per_tok": K, "scoring_func": "sqrtsoftplus", "norm_topk_prob": True,
        "routed_scaling_factor": 1.5, "swiglu_limit": 10.0, "rms_norm_eps": 1e-6, "hc_mult": HC,
        "n_shared_experts": 1, "engram_layer_ids": [ENGRAM_LAYER],
        "engram_num_embeddings": [ROWS], "engram_max_ngram_size": 4, "engram_n_heads": HEADS,
        "engram_head_dim": HD}}
    with open(os.path.join(dirname, "config.json"), "w") as f:
        json.dump(cfg, f)
    return dirname, a
