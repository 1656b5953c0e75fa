"""MoE layer restated in numpy.  Test infrastructure only.

Port semantics (deepseek_v41_mlx/moe.py):
  Gate.__call__     moe.py:58-74    fp32 scores = x.W^T / temp; sqrt(softplus) |
                                    sigmoid | softmax; biased top-k (bias only
                                    selects); weights = unbiased scores at the
                                    picks, / (sum + 1e-20) if normalised, * route_scale
  ClampedSwiGLU     moe.py:30-43    silu(min(gate, L)) * clip(up, -L, L), fp32
  SwitchGLU         moe.py:101-102  (mlx_lm) gate/up projections come back in the
                                    activation dtype (bf16), down takes the fp32 h
  SharedExpert      moe.py:77-93    w1/w3 out bf16, h cast to bf16, w2 out bf16
  MoE.__call__      moe.py:105-112  sum_j w_j * y_j in fp32 (top-k order) + shared,
                                    cast to the input dtype
``round_bf16=False`` keeps every intermediate in fp32 (the "exact" mode the
fp32 1e-5 comparison uses).

Upstream semantics (docs/reference/model.py:792-904) for the a8 prefill form:
weights applied before w2, every linear through act_quant + fp4/fp8 GEMM with
bf16 outputs, expert outputs accumulated in fp32 then the shared expert added.

Ties in top-k pick the lower expert id (torch.topk / mx.argpartition leave
tie order unspecified).
"""

from __future__ import annotations

import numpy as np

from .formats import dequant_fp4, dequant_fp8, round_bf16
from .linear import act_dequant


def _softplus(x):
    return np.logaddexp(x, np.float32(0.0)).astype(np.float32)


def gate_scores(x, gate_w, gate_temp=1.0, score_func="sqrtsoftplus", acc=np.float64):
    """moe.py:59-65 -- activated router scores, float32 [T, E]."""
    s = (np.asarray(x, dtype=acc) @ np.asarray(gate_w, dtype=acc).T).astype(np.float32)
    s = (s / np.float32(gate_temp)).astype(np.float32)
    if score_func == "softmax":
        m = s.max(-1, keepdims=True)
        e = np.exp(s - m)
        return (e / e.sum(-1, keepdims=True)).astype(np.float32)
    if score_func == "sigmoid":
        return (1.0 / (1.0 + np.exp(-s))).astype(np.float32)
    return np.sqrt(_softplus(s)).astype(np.float32)


def topk_lower_index(v: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest per row, descending, ties -> lower index."""
    order = np.argsort(-v, axis=-1, kind="stable")
    return order[..., :k]


def gate(x, gate_w, bias, topk=6, score_func="sqrtsoftplus", gate_temp=1.0,
         norm_topk_prob=True, route_scale=1.5, acc=np.float64):
    """moe.py:58-74 -> (weights f32 [T,k], indices int [T,k], scores f32 [T,E])."""
    scores = gate_scores(x, gate_w, gate_temp, score_func, acc)
    biased = scores + (np.zeros(scores.shape[-1], np.float32) if bias is None
                       else np.asarray(bias, np.float32))
    idx = topk_lower_index(biased.astype(np.float32), topk)
    w = np.take_along_axis(scores, idx, axis=-1).astype(np.float32)
    if norm_topk_prob and topk > 1:
        w = (w / (w.sum(-1, keepdims=True, dtype=np.float32) + np.float32(1e-20))).astype(np.float32)
    w = (w * np.float32(route_scale)).astype(np.float32)
    return w, idx, scores


def topk_margin(x, gate_w, bias, topk, score_func="sqrtsoftplus", gate_temp=1.0):
    """Per token: gap between the k-th and (k+1)-th biased score (for tie tolerance)."""
    scores = gate_scores(x, gate_w, gate_temp, score_func)
    biased = scores + (0 if bias is None else np.asarray(bias, np.float32))
    srt = -np.sort(-biased, axis=-1)
    return srt[:, topk - 1] - srt[:, topk]


def clamped_swiglu(up, gate_v, limit):
    """moe.py:37-43 -- called as activation(x_up, x_gate)."""
    x = np.asarray(up, np.float32)
    g = np.asarray(gate_v, np.float32)
    if limit > 0:
        x = np.clip(x, -limit, limit).astype(np.float32)
        g = np.minimum(g, np.float32(limit)).astype(np.float32)
    with np.errstate(over="ignore"):
        silu = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    return (silu * x).astype(np.float32)


def _mm(a, b, acc):
    return (np.asarray(a, dtype=acc) @ np.asarray(b, dtype=acc).T).astype(np.float32)


def expert_fp4(x_rows, w1, s1, w3, s3, w2, s2, limit, round_bf16_io=True, acc=np.float64):
    """SwitchGLU for one expert on its token rows (port semantics), fp32 [n, D]."""
    W1 = dequant_fp4(w1, s1, "f32")
    W3 = dequant_fp4(w3, s3, "f32")
    W2 = dequant_fp4(w2, s2, "f32")
    g = _mm(x_rows, W1, acc)
    u = _mm(x_rows, W3, acc)
    if round_bf16_io:
        g, u = round_bf16(g), round_bf16(u)
    h = clamped_swiglu(u, g, limit)
    return _mm(h, W2, acc)


def shared_expert_fp8(x, sw1, ss1, sw3, ss3, sw2, ss2, limit, round_bf16_io=True,
                      acc=np.float64):
    """moe.py:85-93 with fp8 32x32 weights (decoded exactly), fp32 [T, D]."""
    W1 = dequant_fp8(sw1, ss1, "f32")
    W3 = dequant_fp8(sw3, ss3, "f32")
    W2 = dequant_fp8(sw2, ss2, "f32")
    g = _mm(x, W1, acc)
    u = _mm(x, W3, acc)
    if round_bf16_io:
        g, u = round_bf16(g), round_bf16(u)
    h = clamped_swiglu(u, g, limit)
    if round_bf16_io:
        h = round_bf16(h)
    y = _mm(h, W2, acc)
    return round_bf16(y) if round_bf16_io else y


def moe_forward(x, p, cfg, round_bf16_io=True, with_shared=True, acc=np.float64, routing=None):
    """moe.py:105-112.  x float32 [T, D] (values of bf16 activations).

    p: dict with gate_w [E,D] (float32 values), gate_bias [E] or None,
       w1,s1,w3,s3 [E,I,D/2],[E,I,D/32]; w2,s2 [E,D,I/2],[E,D,I/32];
       sw1,ss1,sw3,ss3,sw2,ss2 (fp8 shared expert).
    cfg: dict topk, score_func, gate_temp, norm_topk_prob, route_scale, swiglu_limit.
    routing: optional (weights, indices) to use instead of the oracle's own router
    (lets expert math be compared independently of near-tie top-k choices).
    Returns (y float32 [T, D] before the final cast, weights, indices).
    """
    T, D = x.shape
    if routing is None:
        w, idx, _ = gate(x, p["gate_w"], p.get("gate_bias"), cfg["topk"], cfg["score_func"],
                         cfg["gate_temp"], cfg["norm_topk_prob"], cfg["route_scale"], acc)
    else:
        w, idx = (np.asarray(a) for a in routing)
    k = cfg["topk"]
    ys = np.zeros((T, k, D), dtype=np.float32)
    for e in np.unique(idx):
        t_sel, j_sel = np.nonzero(idx == e)
        ye = expert_fp4(x[t_sel], p["w1"][e], p["s1"][e], p["w3"][e], p["s3"][e],
                        p["w2"][e], p["s2"][e], cfg["swiglu_limit"], round_bf16_io, acc)
        ys[t_sel, j_sel] = ye
    y = np.zeros((T, D), dtype=np.float32)
    for j in range(k):                                   # fp32, top-k order
        y = (y + ys[:, j] * w[:, j:j + 1]).astype(np.float32)
    if with_shared:
        sh = shared_expert_fp8(x, p["sw1"], p["ss1"], p["sw3"], p["ss3"], p["sw2"], p["ss2"],
                               cfg["swiglu_limit"], round_bf16_io, acc)
        y = (y + sh).astype(np.float32)
    return y, w, idx


def moe_forward_upstream_a8(x, p, cfg, routing=None, with_shared=True):
    """docs/reference/model.py:889-904 with fp4 experts and fp8 shared expert, a8
    linears (act_quant + block-scaled GEMM), bf16 linear outputs.  ``routing``
    = (weights, indices) replaces the router (e.g. a synthetic skewed routing)."""
    T, D = x.shape
    if routing is None:
        w, idx, _ = gate(x, p["gate_w"], p.get("gate_bias"), cfg["topk"], cfg["score_func"],
                         cfg["gate_temp"], cfg["norm_topk_prob"], cfg["route_scale"])
    else:
        w, idx = (np.asarray(a) for a in routing)
    L = cfg["swiglu_limit"]
    y = np.zeros((T, D), dtype=np.float32)
    xq = act_dequant(round_bf16(x))
    for e in np.unique(idx):
        t_sel, j_sel = np.nonzero(idx == e)
        W1 = dequant_fp4(p["w1"][e], p["s1"][e], "f32")
        W3 = dequant_fp4(p["w3"][e], p["s3"][e], "f32")
        W2 = dequant_fp4(p["w2"][e], p["s2"][e], "f32")
        g = round_bf16(_mm(xq[t_sel], W1, np.float64))
        u = round_bf16(_mm(xq[t_sel], W3, np.float64))
        if L > 0:
            u = np.clip(u, -L, L)
            g = np.minimum(g, np.float32(L))
        h = (g / (1.0 + np.exp(-g))).astype(np.float32) * u
        h = round_bf16(h * w[t_sel, j_sel][:, None])
        ye = round_bf16(_mm(act_dequant(h), W2, np.float64))
        np.add.at(y, t_sel, ye)
    if not with_shared:
        return y.astype(np.float32), w, idx
    W1 = dequant_fp8(p["sw1"], p["ss1"], "f32")
    W3 = dequant_fp8(p["sw3"], p["ss3"], "f32")
    W2 = dequant_fp8(p["sw2"], p["ss2"], "f32")
    g = round_bf16(_mm(xq, W1, np.float64))
    u = round_bf16(_mm(xq, W3, np.float64))
    if L > 0:
        u = np.clip(u, -L, L)
        g = np.minimum(g, np.float32(L))
    h = round_bf16((g / (1.0 + np.exp(-g))).astype(np.float32) * u)
    y = y + round_bf16(_mm(act_dequant(h), W2, np.float64))
    return y.astype(np.float32), w, idx
