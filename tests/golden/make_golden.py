"""Generate the golden fixtures in this directory from the reference's own CPU code.

Run where a checkout of the reference repository is available, naming its root in
$DSV41_REFERENCE:

    DSV41_REFERENCE=<path to the reference checkout> python tests/golden/make_golden.py

What each fixture pins (all from code that ships in the reference repo and
runs without MLX):

* dequant_unit_parity.npz -- the torch half of tests/test_parity.py:348-387
  (seed 11): fp8 32x32, fp4 packed (FP4_TABLE of docs/reference/convert.py:13-15)
  and engram-row decode, exactly as the reference test computes its expected
  values.
* act_quant.npz -- tests/kernel_stub.py act_quant (:47-63), the reference's CPU
  transcription of docs/reference/kernel.py act_quant_kernel, on the inputs of
  tests/test_parity.py:318-345 (seed 3) plus a random bf16 matrix; ue8m0 and
  fp32 scale forms.
* engram_hash.npz -- deepseek_v41_mlx/engram.py EngramHasher (pure numpy; mlx
  is stubbed only so the module imports) on the release config
  (docs/reference/config.json engram_*) with the real compressed-token map
  (engram_token_map.json), called in two chunks; cross-checked against the
  upstream torch NgramHashState.forward (docs/reference/engram.py).
* router_expert.npz -- upstream Gate.forward and Expert.forward
  (docs/reference/model.py:792-851) in fp32 on fp4-decoded weights, plus the
  upstream MoE.forward on a small config (world_size 1).
* engram_embed.npz -- upstream ParallelEngramEmbedding.forward
* engram_gate.npz -- upstream Engram.forward (gated write of the looked-up rows)
  (docs/reference/model.py:312-325), world_size 1.

The fixtures are small (< 1 MB together) and committed; the GPU box never
needs the reference checkout.
"""

from __future__ import annotations

import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("DSV41_REFERENCE", "")


def _setup_imports():
    sys.path.insert(0, os.path.join(REF, "tests"))
    sys.path.insert(0, os.path.join(REF, "docs", "reference"))
    sys.path.insert(0, REF)
    pil = types.ModuleType("PIL")
    pil.Image = types.SimpleNamespace()
    pil.ImageOps = types.SimpleNamespace()
    sys.modules.setdefault("PIL", pil)
    sys.modules.setdefault("tqdm", types.SimpleNamespace(tqdm=lambda x, **k: x,
                                                         trange=lambda *a, **k: range(*a)))
    import kernel_stub
    sys.modules["kernel"] = kernel_stub
    # A minimal stand-in so deepseek_v41_mlx/engram.py imports; only its numpy
    # code (build_layout, compute_hash_multipliers, EngramHasher) is called.
    mlx = types.ModuleType("mlx")
    core = types.ModuleType("mlx.core")
    nn = types.ModuleType("mlx.nn")
    nn.Module = object
    core.__getattr__ = lambda name: object()     # annotations / default args only
    mlx.core, mlx.nn = core, nn
    sys.modules.setdefault("mlx", mlx)
    sys.modules.setdefault("mlx.core", core)
    sys.modules.setdefault("mlx.nn", nn)
    # import the port's submodules without running its package __init__ (which
    # pulls in the MLX model); only config.py and engram.py are used
    pkg = types.ModuleType("deepseek_v41_mlx")
    pkg.__path__ = [os.path.join(REF, "deepseek_v41_mlx")]
    sys.modules.setdefault("deepseek_v41_mlx", pkg)
    return kernel_stub


def golden_dequant():
    """tests/test_parity.py:348-387, torch half, verbatim semantics."""
    import convert as REF_CONVERT
    rng = np.random.default_rng(11)
    OUT, IN = 96, 64
    wb = rng.integers(0, 256, size=(OUT, IN), dtype=np.uint8)
    wb[wb % 128 == 127] = 0
    sb = rng.integers(118, 137, size=(3, 2), dtype=np.uint8)
    tw = torch.from_numpy(wb).view(torch.float8_e4m3fn).float()
    ts = torch.from_numpy(2.0 ** (sb.astype(np.float64) - 127)).float()
    ref8 = (tw * ts.repeat_interleave(32, 0)[:OUT].repeat_interleave(32, 1)[:, :IN])

    pb = rng.integers(0, 256, size=(OUT, IN // 2), dtype=np.uint8)
    s4 = rng.integers(118, 137, size=(OUT, IN // 32), dtype=np.uint8)
    lo, hi = pb & 0x0F, (pb >> 4) & 0x0F
    vals = REF_CONVERT.FP4_TABLE[torch.from_numpy(np.stack([lo, hi], -1)).long()].flatten(1)
    ts4 = torch.from_numpy(2.0 ** (s4.astype(np.float64) - 127)).float()
    ref4 = vals * ts4.repeat_interleave(32, 1)[:, :IN]

    er = torch.from_numpy(wb).view(torch.float8_e4m3fn).float()
    es = rng.integers(118, 137, size=(OUT, IN // 32), dtype=np.uint8)
    tse = torch.from_numpy(2.0 ** (es.astype(np.float64) - 127)).float()
    refr = er * tse.repeat_interleave(32, 1)

    # every e4m3 byte decoded by torch, and the FP4 table itself
    all_e4m3 = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    np.savez_compressed(os.path.join(HERE, "dequant_unit_parity.npz"),
                        wb=wb, sb=sb, ref8=ref8.numpy(), pb=pb, s4=s4, ref4=ref4.numpy(),
                        es=es, refr=refr.numpy(), all_e4m3=all_e4m3,
                        fp4_table=REF_CONVERT.FP4_TABLE.numpy())


def golden_act_quant(kernel_stub):
    rng = np.random.default_rng(3)
    xs = [
        (rng.standard_normal((256, 64)) * np.exp(rng.standard_normal((256, 1)))).astype(np.float32),
        (np.array([0.033203125, -0.033203125, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5,
                   5.0, -5.0, 448.0, 6.0, 1e-9, 0.0, -0.0, 2.0] * 8, dtype=np.float32)
         .reshape(2, 64) * 2.0 ** rng.integers(-8, 9, size=(2, 1)).astype(np.float32)),
    ]
    g = torch.Generator().manual_seed(7)
    xb = (torch.randn(33, 256, generator=g) * 3).to(torch.bfloat16)
    out = {}
    for i, x in enumerate(xs + [xb.float().numpy()]):
        # kernel input is bf16 upstream; round to bf16 first so the fixture is
        # exactly what a bf16 activation produces
        xt = torch.from_numpy(x.copy()).to(torch.bfloat16).float()
        q, s = kernel_stub.act_quant(xt.clone(), 32, "ue8m0", torch.float8_e8m0fnu, False)
        deq = kernel_stub.act_quant(xt.clone(), 32, "ue8m0", torch.float8_e8m0fnu, True)
        qf, sf = kernel_stub.act_quant(xt.clone(), 32, None, torch.float32, False)
        # q returned by the stub is the dequantized fp32 value (q * s); recover codes
        codes = (torch.from_numpy(x.copy()).to(torch.bfloat16).float().reshape(-1, 32)
                 / s.reshape(-1, 1)).clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)
        codesf = (xt.reshape(-1, 32) / sf.reshape(-1, 1)).clamp(-448, 448) \
            .to(torch.float8_e4m3fn).view(torch.uint8)
        out[f"x{i}"] = xt.numpy()
        out[f"codes{i}"] = codes.reshape(xt.shape).numpy()
        out[f"s{i}"] = s.numpy().astype(np.float32)
        out[f"deq{i}"] = deq.numpy()
        out[f"codesf{i}"] = codesf.reshape(xt.shape).numpy()
        out[f"sf{i}"] = sf.numpy().astype(np.float32)
        assert torch.equal(q, deq)
    np.savez_compressed(os.path.join(HERE, "act_quant.npz"), **out)


def golden_engram_hash():
    import deepseek_v41_mlx.engram as PORT
    import engram as UP
    from deepseek_v41_mlx.config import ModelArgs
    cfg = json.load(open(os.path.join(REF, "docs", "reference", "config.json")))
    args = ModelArgs.from_dict(cfg)
    token_map = json.load(open(os.path.join(REF, "engram_token_map.json")))
    if isinstance(token_map, dict):
        token_map = token_map.get("token_map") or token_map.get("map") or list(token_map.values())[0]
    token_map = np.asarray(token_map, dtype=np.int64)
    hasher = PORT.EngramHasher(args, token_map)
    rng = np.random.default_rng(5)
    B, L1, L2, MAXSEQ = 3, 13, 6, 32
    ids = rng.integers(0, len(token_map), size=(B, L1 + L2), dtype=np.int64)
    ids[0, 4] = args.engram_pad_id               # a pad token inside the sequence
    cache = np.zeros((B, MAXSEQ), dtype=np.int64)
    h1 = hasher(ids[:, :L1], 0, cache)
    h2 = hasher(ids[:, L1:], L1, cache)
    # upstream torch NgramHashState.forward on the same inputs
    layout = UP.EngramLayout.from_args(types.SimpleNamespace(**{
        k: getattr(args, k) for k in ("engram_layer_ids", "engram_max_ngram_size",
                                      "engram_n_heads", "engram_vocab_size",
                                      "engram_num_embeddings", "engram_head_dim")}))
    st = UP.NgramHashState.__new__(UP.NgramHashState)
    torch.nn.Module.__init__(st)
    st.layout = layout
    st.pad_id = int(token_map[args.engram_pad_id])
    flat = [[p for g in layer for p in g] for layer in layout.primes]
    offs = [np.cumsum([0, *f[:-1]]) for f in flat]
    st.register_buffer("primes", torch.tensor(layout.primes), persistent=False)
    st.register_buffer("offsets", torch.tensor(np.array(offs)), persistent=False)
    st.register_buffer("multipliers", UP.compute_hash_multipliers(
        layout.layer_ids, layout.max_ngram_size, int(token_map.max()) + 1), persistent=False)
    st.register_buffer("token_map", torch.tensor(token_map), persistent=False)
    st.register_buffer("cache", torch.zeros(B, MAXSEQ, dtype=torch.int64), persistent=False)
    u1 = st.forward(torch.from_numpy(ids[:, :L1]), 0).numpy()
    u2 = st.forward(torch.from_numpy(ids[:, L1:]), L1).numpy()
    assert np.array_equal(u1, h1) and np.array_equal(u2, h2), "port vs upstream hash mismatch"
    np.savez_compressed(os.path.join(HERE, "engram_hash.npz"),
                        ids=ids, L1=L1, h1=h1, h2=h2, cache=cache, primes=hasher.primes,
                        offsets=hasher.offsets, multipliers=hasher.multipliers,
                        pad_id=hasher.pad_id, layer_ids=np.asarray(args.engram_layer_ids),
                        vocab_size=args.engram_vocab_size, n_heads=args.engram_n_heads,
                        max_ngram=args.engram_max_ngram_size,
                        num_embeddings=np.asarray(args.engram_num_embeddings),
                        token_map_sample=token_map[np.unique(ids)], sample_ids=np.unique(ids),
                        token_map_len=len(token_map), token_map_max=int(token_map.max()))


def golden_router_expert():
    import model as M
    M.default_dtype = torch.float32
    torch.manual_seed(0)
    D, I, E, K = 64, 64, 16, 4
    args = M.ModelArgs(dim=D, moe_inter_dim=I, n_routed_experts=E, n_activated_experts=K,
                       n_shared_experts=1, expert_dtype=None, dtype="bf16",
                       score_func="sqrtsoftplus", route_scale=1.5, swiglu_limit=10.0,
                       n_layers=1)
    rng = np.random.default_rng(21)
    T = 24
    x = torch.from_numpy(rng.standard_normal((T, D)).astype(np.float32)).to(torch.bfloat16).float()
    gw = torch.from_numpy((rng.standard_normal((E, D)) / np.sqrt(D)).astype(np.float32)) \
        .to(torch.bfloat16).float()
    gb = torch.from_numpy((rng.standard_normal(E) * 0.01).astype(np.float32))
    moe = M.MoE(0, args)
    moe.gate.weight.data.copy_(gw)
    moe.gate.bias.data.copy_(gb)
    w, idx = moe.gate(x)
    # fp4 experts decoded exactly into the fp32 Expert linears
    import convert as REF_CONVERT

    def fp4(out, inn):
        pk = rng.integers(0, 256, size=(out, inn // 2), dtype=np.uint8)
        sc = rng.integers(120, 129, size=(out, inn // 32), dtype=np.uint8)
        lo, hi = pk & 0x0F, (pk >> 4) & 0x0F
        v = REF_CONVERT.FP4_TABLE[torch.from_numpy(np.stack([lo, hi], -1)).long()].flatten(1)
        v = v * torch.from_numpy(2.0 ** (sc.astype(np.float64) - 127)).float().repeat_interleave(32, 1)
        return pk, sc, v

    packs = {"w1": [], "s1": [], "w3": [], "s3": [], "w2": [], "s2": []}
    for e in range(E):
        for name, (o, i_) in (("w1", (I, D)), ("w3", (I, D)), ("w2", (D, I))):
            pk, sc, v = fp4(o, i_)
            packs[name].append(pk)
            packs["s" + name[1]].append(sc)
            getattr(moe.experts[e], name).weight.data.copy_(v)

    def fp8(out, inn):
        wb = rng.integers(0, 256, size=(out, inn), dtype=np.uint8)
        wb[wb % 128 == 127] = 0
        sc = rng.integers(118, 128, size=((out + 31) // 32, (inn + 31) // 32), dtype=np.uint8)
        tw = torch.from_numpy(wb).view(torch.float8_e4m3fn).float()
        ts = torch.from_numpy(2.0 ** (sc.astype(np.float64) - 127)).float()
        return wb, sc, tw * ts.repeat_interleave(32, 0)[:out].repeat_interleave(32, 1)[:, :inn]

    sh = {}
    for name, (o, i_) in (("sw1", (I, D)), ("sw3", (I, D)), ("sw2", (D, I))):
        wb, sc, v = fp8(o, i_)
        sh[name], sh["ss" + name[2]] = wb, sc
        getattr(moe.shared_experts, name[1:]).weight.data.copy_(v)
    e0 = int(idx[0, 0])
    y_expert = moe.experts[e0](x[:5]).detach().numpy()          # weights=None path
    y_moe = moe(x).detach().numpy()
    np.savez_compressed(os.path.join(HERE, "router_expert.npz"),
                        x=x.numpy(), gate_w=gw.numpy(), gate_bias=gb.numpy(),
                        weights=w.detach().numpy(), indices=idx.numpy(), e0=e0, y_expert=y_expert,
                        y_moe=y_moe, topk=K, swiglu_limit=10.0, route_scale=1.5,
                        **{k: np.stack(v) for k, v in packs.items()}, **sh)


def golden_engram_embed():
    import model as M
    M.world_size, M.rank = 1, 0
    rng = np.random.default_rng(9)
    rows, d = 300, 256
    emb = M.ParallelEngramEmbedding(rows, d)
    wb = rng.integers(0, 256, size=(rows, d), dtype=np.uint8)
    wb[wb % 128 == 127] = 0
    sc = rng.integers(115, 128, size=(rows, d // 32), dtype=np.uint8)
    emb.weight.data.copy_(torch.from_numpy(wb).view(torch.float8_e4m3fn))
    emb.scale.data.copy_(torch.from_numpy(sc).view(torch.float8_e8m0fnu))
    idx = torch.from_numpy(rng.integers(0, rows, size=(5, 24), dtype=np.int64))
    out = emb(idx).float().detach().numpy()
    np.savez_compressed(os.path.join(HERE, "engram_embed.npz"), table=wb, scale=sc,
                        idx=idx.numpy(), out=out)


def golden_engram_gate():
    """upstream Engram.forward (docs/reference/model.py:344-365) in fp32 with the row lookup
    replaced by fixed rows: kv = wkv(rows), the per-(token, hc copy) normalised gate and the
    gated write, with and without a token mask.  Inputs are bf16-representable."""
    import model as M
    M.default_dtype = torch.float32
    M.world_size, M.rank = 1, 0
    rng = np.random.default_rng(31)
    D, hc, hd, B, L = 64, 4, 16, 2, 5
    layout = types.SimpleNamespace(layer_ids=(1,), num_embeddings=(100,), head_dim=hd,
                                   max_ngram_size=4, n_heads=2)
    cols = (layout.max_ngram_size - 1) * layout.n_heads
    args = M.ModelArgs(dim=D, n_layers=1, hc_mult=hc, norm_eps=1e-6)
    eg = M.Engram(args, 1, layout)

    def bf(a):
        return torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).float()

    eg.wkv.weight.data.copy_(bf(rng.standard_normal(((hc + 1) * D, cols * hd)) / np.sqrt(cols * hd)))
    eg.q_weight.data.copy_(bf(1.0 + 0.1 * rng.standard_normal((hc, D))))
    eg.k_weight.data.copy_(bf(1.0 + 0.1 * rng.standard_normal((hc, D))))
    rows = bf(rng.standard_normal((B, L, cols, hd)))

    class Rows(torch.nn.Module):
        def forward(self, ids):
            return rows

    eg._modules["embed"] = Rows()
    x = bf(rng.standard_normal((B, L, hc, D)))
    ids = torch.zeros((B, L, cols), dtype=torch.int64)
    mask = torch.from_numpy(rng.random((B, L)) > 0.3)
    with torch.no_grad():
        kv = eg.wkv(rows.flatten(-2))
        out = eg(x, ids)
        out_m = eg(x, ids, mask)
    np.savez_compressed(os.path.join(HERE, "engram_gate.npz"), x=x.numpy(), rows=rows.numpy(),
                        wkv=eg.wkv.weight.detach().numpy(), kv=kv.numpy(),
                        q_weight=eg.q_weight.detach().numpy(),
                        k_weight=eg.k_weight.detach().numpy(), eps=eg.eps,
                        clamp=eg.clamp_value, out=out.numpy(), mask=mask.numpy(),
                        out_masked=out_m.numpy())


def main():
    if not REF or not os.path.isdir(os.path.join(REF, "deepseek_v41_mlx")):
        sys.exit("set DSV41_REFERENCE to the root of a checkout of the reference repository")
    torch.set_default_dtype(torch.float32)
    ks = _setup_imports()
    golden_dequant()
    golden_act_quant(ks)
    golden_engram_hash()
    golden_router_expert()
    golden_engram_embed()
    golden_engram_gate()
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
