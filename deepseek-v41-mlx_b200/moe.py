"""MoE on the GPU -- drop-in for deepseek_v41_mlx/moe.py.

Same classes and attributes as the reference (moe.py:30-112):

* ``ClampedSwiGLU(limit)(x, gate)``          -- silu(min(gate, L)) * clip(x, -L, L), fp32
* ``Gate(args)(x) -> (weights, indices)``    -- sqrt-softplus router, biased top-k
* ``SharedExpert(dim, inter, limit)(x)``     -- fp8 32x32 weights (release format)
* ``MoE(args)(x)``                           -- routed fp4 experts + shared expert;
  ``MoE.gate`` and ``MoE.experts(xf, indices) -> [T, k, dim]`` stay separately
  callable (scripts/reap_calibrate.py:47-65 patches ``MoE.__call__`` around them).

Weights are the native release tensors, not converted ones: routed experts
``experts.{gate,up,down}_proj.weight`` uint8 [E, out, in/2] (e2m1 pairs) with
``.scales`` uint8 [E, out, in/32] (ue8m0); shared expert ``w1/w2/w3.weight``
e4m3 [out, in] with ``.scale`` ue8m0 [ceil(out/32), ceil(in/32)]; the router
``gate.weight`` bf16 [E, dim], ``gate.bias`` f32 [E].

Numerics follow the port (``round_bf16=True``: gate/up outputs and the shared
expert's intermediates rounded to bf16 as MLX produces them) or keep every
intermediate in fp32 (``round_bf16=False``).
"""

from __future__ import annotations

import ctypes as C
import gc

from . import _lib as L


def _torch():
    return L.torch()


class ClampedSwiGLU:
    """moe.py:30-43 -- called as activation(x_up, x_gate)."""

    def __init__(self, limit: float = 0.0):
        self.limit = limit

    def __call__(self, x, gate):
        t = _torch()
        x = L.cuda_tensor(x, "x").float()
        gate = L.cuda_tensor(gate, "gate").float()
        if self.limit > 0:
            x = t.clamp(x, -self.limit, self.limit)
            gate = t.clamp(gate, max=self.limit)
        return t.nn.functional.silu(gate) * x


class Gate:
    """moe.py:46-74."""

    def __init__(self, args):
        t = _torch()
        self.topk = args.n_activated_experts
        self.score_func = args.score_func
        self.gate_temp = args.gate_temp
        self.norm_topk_prob = args.norm_topk_prob
        self.route_scale = args.route_scale
        self.weight = t.zeros((args.n_routed_experts, args.dim), dtype=t.bfloat16)
        self.bias = t.zeros((args.n_routed_experts,), dtype=t.float32)
        self.bias_vl = t.zeros((args.n_routed_experts,), dtype=t.float32)

    def __call__(self, x):
        t = _torch()
        xt = L.cuda_tensor(x, "x")
        if xt.dtype != t.bfloat16:
            xt = xt.to(t.bfloat16)
        w = L.cuda_tensor(self.weight, "gate.weight").to(t.bfloat16)
        b = L.cuda_tensor(self.bias, "gate.bias").float()
        D = xt.shape[-1]
        xf = xt.reshape(-1, D)
        T, E = xf.shape[0], w.shape[0]
        weights = t.empty((T, self.topk), dtype=t.float32, device=xf.device)
        indices = t.empty((T, self.topk), dtype=t.int32, device=xf.device)
        ws = L.workspace(L.load().dsv41_moe_route_workspace_size(T, D, E), xf.device)
        L.call("dsv41_moe_route", L.ptr(xf), T, D, L.ptr(w), L.ptr(b), E, self.topk,
               L.SCORE_FUNCS[self.score_func], float(self.gate_temp), int(self.norm_topk_prob),
               float(self.route_scale), L.ptr(weights), L.ptr(indices), L.ptr(ws), ws.numel(),
               L.stream_of(xf))
        shp = tuple(xt.shape[:-1]) + (self.topk,)
        return weights.reshape(shp), indices.reshape(shp)


class _Proj:
    """One stacked projection (weight + scales)."""

    def __init__(self, weight=None, scales=None):
        self.weight = weight
        self.scales = scales


class SwitchGLU:
    """Stacked fp4 experts (the role of mlx_lm SwitchGLU at moe.py:101-102)."""

    def __init__(self, dim, inter, n_experts, limit):
        self.dim, self.inter, self.n_experts = dim, inter, n_experts
        self.activation = ClampedSwiGLU(limit)
        self.gate_proj, self.up_proj, self.down_proj = _Proj(), _Proj(), _Proj()
        self._owner = None

    def __call__(self, x, indices):
        """x [T, dim] bf16, indices [T, k] -> unweighted expert outputs [T, k, dim] fp32."""
        return self._owner._experts(x, indices)


class SharedExpert:
    """moe.py:77-93 with fp8 32x32 weights (w1 gate, w3 up, w2 down)."""

    def __init__(self, dim, inter_dim, limit=0.0):
        self.dim, self.inter, self.limit = dim, inter_dim, limit
        self.w1, self.w2, self.w3 = _Proj(), _Proj(), _Proj()

    def __call__(self, x):
        from .linear import linear_fp8
        t = _torch()
        xt = L.cuda_tensor(x, "x")
        dtype = xt.dtype
        g = linear_fp8(xt, self.w1.weight, self.w1.scales, out_dtype=dtype).float()
        u = linear_fp8(xt, self.w3.weight, self.w3.scales, out_dtype=dtype).float()
        if self.limit > 0:
            u = t.clamp(u, -self.limit, self.limit)
            g = t.clamp(g, max=self.limit)
        h = t.nn.functional.silu(g) * u
        return linear_fp8(h.to(dtype), self.w2.weight, self.w2.scales, out_dtype=dtype)


class MoE:
    """moe.py:96-112.  Up to ``a16_min_tokens`` tokens a call (default 2048) run on the
    decode engine; larger calls run the same numerics on the tensor cores
    (``prefill_a16``), which is faster there (measured on B200 with the release shapes:
    T=2048 7.6 vs 7.7 ms, T=4096 13.8 vs 8.6 ms) and has no token limit.

    With ``cuda_graph=True`` (default) each (tokens, output dtype, device) shape is
    captured once into a CUDA graph (router, plan, expert kernels, shared expert
    on a forked stream, combine) and replayed; the graph owns its input/output
    buffers and workspace and is rebuilt if any weight tensor is replaced or modified.
    Outputs are fresh tensors (copies of the graph's buffers), as the reference's
    functional API returns new arrays.

    With ``pack_decode_scales=True`` (default, when dim and moe_inter_dim are
    multiples of 256) the routed experts' ue8m0 scales are rearranged once into the
    decode-packed layout (``dsv41_moe_decode_pack``: one contiguous block per 64-row
    tile and K stage) and rebuilt when a scale tensor changes; the decode kernels then
    fetch each stage's scales with one bulk copy.  With packed scales the routed down
    projection runs two 64-row tiles of an expert per work item once those items fill a
    wave of CTAs; ``row_pair_down=False`` keeps it on single tiles (same bits).
    """

    def __init__(self, args, round_bf16: bool = True, cuda_graph: bool = True,
                 pack_decode_scales: bool = True, row_pair_down: bool = True,
                 a16_min_tokens: int = 2048):
        self.args = args
        self.a16_min_tokens = a16_min_tokens
        self.dim = args.dim
        self.gate = Gate(args)
        self.experts = SwitchGLU(args.dim, args.moe_inter_dim, args.n_routed_experts,
                                 args.swiglu_limit)
        self.experts._owner = self
        self.shared_experts = SharedExpert(args.dim, args.moe_inter_dim, args.swiglu_limit)
        self.round_bf16 = round_bf16
        self.cuda_graph = cuda_graph
        self.pack_decode_scales = pack_decode_scales
        self.row_pair_down = row_pair_down
        self._dpack = None
        self._dpack_key = None
        self._ws = None
        self._graphs = {}
        self._graph_sig = None

    def _sig(self):
        e, s = self.experts, self.shared_experts
        objs = (self.gate.weight, self.gate.bias, e.gate_proj.weight, e.gate_proj.scales,
                e.up_proj.weight, e.up_proj.scales, e.down_proj.weight, e.down_proj.scales,
                s.w1.weight, s.w1.scales, s.w3.weight, s.w3.scales, s.w2.weight, s.w2.scales)
        return (self.pack_decode_scales, self.row_pair_down, self.round_bf16) + tuple(
            (id(o), o.data_ptr() if hasattr(o, "data_ptr") else 0, getattr(o, "_version", 0))
            for o in objs)

    def _decode_into(self, xf, y, weights, indices, W, ws, cfg):
        T = xf.shape[0]
        L.call("dsv41_moe_decode", C.byref(cfg), C.byref(W), L.ptr(xf), T, L.dtype_code(y.dtype),
               L.ptr(y), L.ptr(weights), L.ptr(indices), L.ptr(ws), ws.numel(), L.stream_of(xf))

    def _graph_call(self, xf, odt, with_routing=True):
        t = _torch()
        sig = self._sig()
        if sig != self._graph_sig:
            self._graphs = {}
            self._graph_sig = sig
        T = xf.shape[0]
        key = (T, odt, xf.device)
        ent = self._graphs.get(key)
        if ent is None:
            k = self.args.n_activated_experts
            sx = t.empty_like(xf)
            sy = t.empty((T, self.dim), dtype=odt, device=xf.device)
            sw = t.empty((T, k), dtype=t.float32, device=xf.device)
            si = t.empty((T, k), dtype=t.int32, device=xf.device)
            cfg, W = self._decode_args()
            ws = L.workspace(L.load().dsv41_moe_decode_workspace_size(C.byref(cfg), T), xf.device)
            keep = list(self._keep)
            sx.copy_(xf)
            side = t.cuda.Stream(device=xf.device)
            side.wait_stream(t.cuda.current_stream(xf.device))
            with t.cuda.stream(side):                      # warm-up outside capture
                self._decode_into(sx, sy, sw, si, W, ws, cfg)
            t.cuda.current_stream(xf.device).wait_stream(side)
            g = t.cuda.CUDAGraph()
            # dead Python cycles that own CUDA graphs or events are collected now: a collection
            # inside the capture would destroy them there and invalidate the capture
            gc_on = gc.isenabled()
            gc.collect()
            gc.disable()
            try:
                with t.cuda.graph(g):
                    self._decode_into(sx, sy, sw, si, W, ws, cfg)
            finally:
                if gc_on:
                    gc.enable()
            ent = (g, sx, sy, sw, si, ws, W, keep, cfg)
            self._graphs[key] = ent
        g, sx, sy, sw, si = ent[:5]
        sx.copy_(xf)
        g.replay()
        if not with_routing:
            return sy.clone(), None, None
        return sy.clone(), sw.clone(), si.clone()

    # -- plumbing --------------------------------------------------------------
    def _cfg(self, flags=0):
        a = self.args
        return L.MoeConfig(dim=a.dim, inter=a.moe_inter_dim, n_experts=a.n_routed_experts,
                           topk=a.n_activated_experts, score_func=L.SCORE_FUNCS[a.score_func],
                           gate_temp=float(a.gate_temp), norm_topk_prob=int(a.norm_topk_prob),
                           route_scale=float(a.route_scale), swiglu_limit=float(a.swiglu_limit),
                           flags=(L.MOE_ROUND_BF16 if self.round_bf16 else 0)
                           | (0 if self.row_pair_down else L.MOE_NO_ROWPAIR) | flags)

    def _weights(self):
        t = _torch()
        self._keep = []

        def p(a, conv=None):
            if a is None:
                return None
            v = L.cuda_tensor(a)
            if conv is not None:
                v = conv(v)
            self._keep.append(v)
            return L.ptr(v)

        e, s = self.experts, self.shared_experts
        return L.MoeWeights(
            gate_w=p(self.gate.weight, lambda v: v.to(t.bfloat16)),
            gate_bias=p(self.gate.bias, lambda v: v.float()),
            w1=p(e.gate_proj.weight, L.u8), s1=p(e.gate_proj.scales, L.u8),
            w3=p(e.up_proj.weight, L.u8), s3=p(e.up_proj.scales, L.u8),
            w2=p(e.down_proj.weight, L.u8), s2=p(e.down_proj.scales, L.u8),
            sw1=p(s.w1.weight, L.u8), ss1=p(s.w1.scales, L.u8),
            sw3=p(s.w3.weight, L.u8), ss3=p(s.w3.scales, L.u8),
            sw2=p(s.w2.weight, L.u8), ss2=p(s.w2.scales, L.u8))

    def _decode_pack(self, cfg, W):
        """The routed experts' scales in the decode-packed layout, or None when the shapes
        do not allow it (dim and inter must be multiples of 256)."""
        a = self.args
        e = self.experts
        if (not self.pack_decode_scales or a.dim % 256 or a.moe_inter_dim % 256
                or e.gate_proj.scales is None):
            return None
        srcs = [L.cuda_tensor(p.scales) for p in (e.gate_proj, e.up_proj, e.down_proj)]
        key = tuple((s.data_ptr(), s._version, tuple(s.shape)) for s in srcs)
        if self._dpack_key != key:
            n = L.load().dsv41_moe_decode_pack_size(C.byref(cfg))
            buf = L.workspace(n, srcs[0].device)
            L.call("dsv41_moe_decode_pack", C.byref(cfg), C.byref(W), L.ptr(buf), n,
                   L.stream_of(buf))
            self._dpack, self._dpack_key = buf, key
        return self._dpack

    def _decode_args(self, flags=0):
        """(config, weights) for the decode entries, with the decode-packed scales when
        they apply."""
        cfg = self._cfg(flags)
        W = self._weights()
        pk = self._decode_pack(cfg, W)
        if pk is not None:
            a = self.args
            gu = a.n_routed_experts * a.moe_inter_dim * (a.dim // 32)
            base = L.ptr(pk)
            W.s1, W.s3, W.s2 = base, base + gu, base + 2 * gu
            cfg.flags |= L.MOE_PACKED_SCALES
            self._keep.append(pk)
        return cfg, W

    def _workspace(self, cfg, T, device):
        need = L.load().dsv41_moe_decode_workspace_size(C.byref(cfg), T)
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            self._ws = L.workspace(need, device)
        return self._ws

    def _experts(self, x, indices):
        t = _torch()
        xt = L.cuda_tensor(x, "x").to(t.bfloat16)
        xf = xt.reshape(-1, self.dim)
        idx = L.cuda_tensor(indices, "indices").to(t.int32).reshape(xf.shape[0], -1)
        T, k = idx.shape
        cfg, W = self._decode_args(L.MOE_NO_SHARED)
        y = t.empty((T, k, self.dim), dtype=t.float32, device=xf.device)
        ws = self._workspace(cfg, T, xf.device)
        L.call("dsv41_moe_experts", C.byref(cfg), C.byref(W), L.ptr(xf), T, L.ptr(idx), L.ptr(y),
               L.ptr(ws), ws.numel(), L.stream_of(xf))
        return y

    def __call__(self, x, with_routing: bool = False, out_dtype=None):
        t = _torch()
        xt = L.cuda_tensor(x, "x")
        shape = xt.shape
        xf = xt.to(t.bfloat16).reshape(-1, self.dim)
        T = xf.shape[0]
        odt = out_dtype or (t.float32 if xt.dtype == t.float32 else t.bfloat16)
        if T > self.a16_min_tokens:
            weights, indices = self.gate(xf)
            y = self.prefill_a16(xf, weights=weights, indices=indices, out_dtype=odt)
            y = y.reshape(shape)
            return (y, weights, indices) if with_routing else y
        if self.cuda_graph and not t.cuda.is_current_stream_capturing():
            y, weights, indices = self._graph_call(xf, odt, with_routing)
            y = y.reshape(shape)
            return (y, weights, indices) if with_routing else y
        cfg, W = self._decode_args()
        y = t.empty((T, self.dim), dtype=odt, device=xf.device)
        k = self.args.n_activated_experts
        weights = t.empty((T, k), dtype=t.float32, device=xf.device)
        indices = t.empty((T, k), dtype=t.int32, device=xf.device)
        ws = self._workspace(cfg, T, xf.device)
        L.call("dsv41_moe_decode", C.byref(cfg), C.byref(W), L.ptr(xf), T, L.dtype_code(odt),
               L.ptr(y), L.ptr(weights), L.ptr(indices), L.ptr(ws), ws.numel(), L.stream_of(xf))
        y = y.reshape(shape)
        return (y, weights, indices) if with_routing else y

    # -- prefill, upstream a8 numerics ---------------------------------------
    def prefill_a8(self, x, weights=None, indices=None, out_dtype=None, topk=None,
                   shared=True, routed=True):
        """The layer as upstream runs it (docs/reference/model.py:889-904): every
        linear in a8 form (act_quant + block-scaled GEMM, bf16 outputs), routed
        experts as grouped GEMMs on tcgen05 block-scaled MMA.  Routing is computed
        by the router unless ``weights``/``indices`` [T, topk] are given.
        ``routed=False``: the shared expert alone; ``shared=False``: the routed
        experts alone; ``topk`` overrides the config (1 = every row is one pair, the
        owner side of expert parallelism)."""
        t = _torch()
        xt = L.cuda_tensor(x, "x")
        shape = xt.shape
        xf = xt.to(t.bfloat16).reshape(-1, self.dim).contiguous()
        T = xf.shape[0]
        odt = out_dtype or (t.float32 if xt.dtype == t.float32 else t.bfloat16)
        se = self.shared_experts
        has_shared = shared and se is not None and se.w1.weight is not None
        flags = (0 if has_shared else L.MOE_NO_SHARED) | (0 if routed else L.MOE_SHARED_ONLY)
        cfg = self._cfg(flags)
        if topk is not None:
            cfg.topk = int(topk)
        W = self._weights()
        given = indices is not None or not routed
        if indices is not None:
            idx = L.cuda_tensor(indices, "indices").to(t.int32).reshape(T, -1).contiguous()
            wts = L.cuda_tensor(weights, "weights").float().reshape(T, -1).contiguous()
        packed = self._packed_scales(cfg, W, xf.device)
        need = L.load().dsv41_moe_prefill_workspace_size(C.byref(cfg), T, 1 if given else 0, 1)
        ws = L.workspace(need, xf.device)
        y = t.empty((T, self.dim), dtype=odt, device=xf.device)
        has_idx = indices is not None
        L.call("dsv41_moe_prefill", C.byref(cfg), C.byref(W), L.ptr(packed), L.ptr(xf), T,
               L.ptr(wts) if has_idx else None, L.ptr(idx) if has_idx else None,
               L.dtype_code(odt), L.ptr(y), L.ptr(ws), ws.numel(), L.stream_of(xf))
        return y.reshape(shape)

    # -- prefill, the port's numerics ----------------------------------------
    def prefill_a16(self, x, weights=None, indices=None, out_dtype=None, shared=True,
                    routed=True):
        """The layer at prefill sizes as the port computes it (moe.py:96-112): bf16
        activations times the release's fp4 experts and fp8 shared expert decoded exactly to
        bf16, on the tensor cores (``dsv41_moe_prefill_a16``); gate/up outputs and the shared
        expert's intermediates rounded to bf16 when ``round_bf16`` (else fp32 throughout),
        the down projection on the fp32 SwiGLU output, expert outputs weighted and summed in
        top-k order.  Routing is computed by the router unless ``weights``/``indices``
        [T, topk] are given; ``shared=False`` / ``routed=False`` leave one part out."""
        t = _torch()
        xt = L.cuda_tensor(x, "x")
        shape = xt.shape
        xf = xt.to(t.bfloat16).reshape(-1, self.dim).contiguous()
        T = xf.shape[0]
        odt = out_dtype or (t.float32 if xt.dtype == t.float32 else t.bfloat16)
        se = self.shared_experts
        has_shared = shared and se is not None and se.w1.weight is not None
        flags = (0 if has_shared else L.MOE_NO_SHARED) | (0 if routed else L.MOE_SHARED_ONLY)
        cfg = self._cfg(flags)
        W = self._weights()
        has_idx = indices is not None
        if has_idx:
            idx = L.cuda_tensor(indices, "indices").to(t.int32).reshape(T, -1).contiguous()
            wts = L.cuda_tensor(weights, "weights").float().reshape(T, -1).contiguous()
        need = L.load().dsv41_moe_prefill_a16_workspace_size(C.byref(cfg), T, 1 if has_idx else 0)
        ws = L.workspace(need, xf.device)
        y = t.empty((T, self.dim), dtype=odt, device=xf.device)
        L.call("dsv41_moe_prefill_a16", C.byref(cfg), C.byref(W), L.ptr(xf), T,
               L.ptr(wts) if has_idx else None, L.ptr(idx) if has_idx else None,
               L.dtype_code(odt), L.ptr(y), L.ptr(ws), ws.numel(), L.stream_of(xf))
        return y.reshape(shape)

    def _packed_scales(self, cfg, W, device):
        """Expert scales in the tensor-core layout, rebuilt when a scale tensor changes."""
        e, se = self.experts, self.shared_experts
        projs = [p for p in (e.gate_proj, e.up_proj, e.down_proj) if p.scales is not None]
        if se is not None:
            projs += [p for p in (se.w1, se.w3, se.w2) if p.scales is not None]
        srcs = [L.cuda_tensor(p.scales) for p in projs]
        key = tuple((s.data_ptr(), s._version, tuple(s.shape)) for s in srcs)
        if getattr(self, "_pack_key", None) != key:
            n = L.load().dsv41_moe_prefill_pack_size(C.byref(cfg))
            self._pack = L.workspace(n, device)
            L.call("dsv41_moe_prefill_pack", C.byref(cfg), C.byref(W), L.ptr(self._pack), n,
                   L.stream_of(self._pack))
            self._pack_key = key
        return self._pack
