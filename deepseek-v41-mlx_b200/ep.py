"""Expert parallelism for the MoE layer over torch.distributed (NCCL on GPUs).

Upstream shards experts by rank (rank r owns experts [r*E/ws, (r+1)*E/ws),
docs/reference/model.py:854-867) but lets every rank see every token and sums
the partial outputs with an fp32 all_reduce (model.py:895-902).  Here each rank
keeps its own tokens and only the (token, expert) pairs travel:

1. route locally (router weights are replicated);
2. dispatch: pairs are ordered by owning rank, the per-rank counts are exchanged
   with one all_to_all, then the bf16 token rows and the owner-local expert ids
   move with all_to_all_single;
3. the owner runs its experts on the received rows (the fused decode kernels,
   each received row being one pair);
4. combine: the fp32 expert outputs return with the mirror all_to_all_single and
   are summed per token in top-k order with the routing weights, then the shared
   expert (computed locally) is added -- the same order of fp32 operations as the
   single-GPU layer.

The exchange logic is plain torch and runs with gloo on CPU (tests) or NCCL on
GPUs; the expert computation is a callable so the CPU tests can inject a torch
reference while the GPU path calls libdsv41q.
"""

from __future__ import annotations

import ctypes as C

from . import _lib as L


def owner_of(indices, experts_per_rank: int):
    return indices // experts_per_rank


def plan_dispatch(indices, world: int, experts_per_rank: int):
    """indices int [T, k] -> (order, send_counts) with pairs ordered by owner rank
    (stable, row-major over [T, k])."""
    t = L.torch()
    flat = indices.reshape(-1).to(t.int64)
    owner = owner_of(flat, experts_per_rank)
    order = t.argsort(owner * flat.numel() + t.arange(flat.numel(), device=flat.device))
    counts = t.bincount(owner, minlength=world)
    return order, counts


def exchange_counts(dist, send_counts, group=None):
    t = L.torch()
    recv = t.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts, group=group)
    return recv


def dispatch(dist, x, indices, world, experts_per_rank, group=None, weights=None):
    """-> (recv_rows [R, D], recv_local_expert [R], order, send_counts, recv_counts) and, when
    ``weights`` [T, k] is given, the pairs' routing weights recv_w [R] last."""
    t = L.torch()
    D = x.shape[-1]
    k = indices.shape[-1]
    order, send_counts = plan_dispatch(indices, world, experts_per_rank)
    recv_counts = exchange_counts(dist, send_counts, group)
    tok = order // k
    send_rows = x.reshape(-1, D).index_select(0, tok).contiguous()
    send_exp = (indices.reshape(-1).to(t.int64).index_select(0, order) % experts_per_rank).to(t.int32)
    sc = send_counts.tolist()
    rc = recv_counts.tolist()
    R = int(sum(rc))
    recv_rows = t.empty((R, D), dtype=x.dtype, device=x.device)
    recv_exp = t.empty((R,), dtype=t.int32, device=x.device)
    dist.all_to_all_single(recv_rows, send_rows, rc, sc, group=group)
    dist.all_to_all_single(recv_exp, send_exp, rc, sc, group=group)
    if weights is None:
        return recv_rows, recv_exp, order, sc, rc
    send_w = weights.reshape(-1).float().index_select(0, order).contiguous()
    recv_w = t.empty((R,), dtype=t.float32, device=x.device)
    dist.all_to_all_single(recv_w, send_w, rc, sc, group=group)
    return recv_rows, recv_exp, order, sc, rc, recv_w


def combine(dist, y_recv, order, send_counts, recv_counts, T, k, group=None):
    """Return the owners' fp32 outputs to their pairs: -> Y [T, k, D] (unweighted)."""
    t = L.torch()
    D = y_recv.shape[-1]
    back = t.empty((sum(send_counts), D), dtype=y_recv.dtype, device=y_recv.device)
    dist.all_to_all_single(back, y_recv.contiguous(), send_counts, recv_counts, group=group)
    Y = t.empty((T * k, D), dtype=y_recv.dtype, device=y_recv.device)
    Y.index_copy_(0, order, back)
    return Y.reshape(T, k, D)


def ascending_sum(Y, indices, shared=None):
    """sum over j of Y[t, j] in ascending expert-id order (fp32), then + shared: the order of
    upstream's expert loop (docs/reference/model.py:895-900) and of the single-GPU prefill."""
    t = L.torch()
    order = t.argsort(indices.to(t.int64), dim=1, stable=True)
    Ys = t.take_along_dim(Y, order[:, :, None], dim=1)
    acc = t.zeros(Y.shape[0], Y.shape[2], dtype=t.float32, device=Y.device)
    for j in range(Y.shape[1]):
        acc = acc + Ys[:, j].float()
    if shared is not None:
        acc = acc + shared.float()
    return acc


def weighted_sum(Y, weights, shared=None):
    """sum_j w[t, j] * Y[t, j] in j order (fp32), + shared: the single-GPU combine."""
    t = L.torch()
    acc = t.zeros(Y.shape[0], Y.shape[2], dtype=t.float32, device=Y.device)
    for j in range(Y.shape[1]):
        acc = acc + Y[:, j].float() * weights[:, j:j + 1].float()
    if shared is not None:
        acc = acc + shared.float()
    return acc


class EPMoE:
    """MoE layer with routed experts sharded over the process group.

    ``local`` is a single-GPU ``moe.MoE`` holding this rank's experts (ids
    renumbered 0 .. E/ws-1) plus the replicated router and shared expert.
    """

    def __init__(self, local, world: int, rank: int, n_experts: int, group=None,
                 max_tokens: int = 256, p2p: bool = True):
        import torch.distributed as dist
        self.dist = dist
        self.local = local
        self.world, self.rank = world, rank
        self.E = n_experts
        self.epr = n_experts // world
        self.group = group
        self.local_active = []
        self.track = False
        self.max_tokens = max_tokens      # decode tokens per rank and call (peer-memory path)
        self.p2p = p2p
        self._ctx = None
        self._ws = None

    # ---------------------------------------------------------------- GPU path
    @staticmethod
    def _random_layer(q, torch, dev, n_experts, D, I, topk, seed):
        """An empty MoE layer of ``n_experts`` experts and the generator that draws the parts
        every rank holds alike (the router over all experts and the shared expert)."""
        import types
        g = torch.Generator(device=dev).manual_seed(seed)
        args = types.SimpleNamespace(n_activated_experts=topk, score_func="sqrtsoftplus",
                                     gate_temp=1.0, norm_topk_prob=True, route_scale=1.5,
                                     n_routed_experts=n_experts, dim=D, moe_inter_dim=I,
                                     swiglu_limit=10.0)
        m = q.moe.MoE(args, round_bf16=True, cuda_graph=False)
        return m, g

    @staticmethod
    def _draw_replicated(torch, dev, m, g, E, D, I):
        gate_w = (torch.randn(E, D, device=dev, generator=g) * D ** -0.5).to(torch.bfloat16)
        gate_b = torch.randn(E, device=dev, generator=g) * 0.01
        for key, (n, k) in (("1", (I, D)), ("3", (I, D)), ("2", (D, I))):
            w = torch.randint(0, 256, (n, k), dtype=torch.uint8, device=dev, generator=g)
            w[(w & 0x7F) == 0x7F] = 0
            pr = getattr(m.shared_experts, "w" + key)
            pr.weight = w
            pr.scales = torch.randint(118, 128, (n // 32, k // 32), dtype=torch.uint8, device=dev,
                                      generator=g)
        return gate_w, gate_b

    @staticmethod
    def _draw_shard(torch, dev, rank, epr, D, I, seed):
        """Rank ``rank``'s experts: {projection: (weight, scales)}, from its own generator."""
        gl = torch.Generator(device=dev).manual_seed(seed + 1000 + rank)
        out = {}
        for name, (n, k) in (("gate_proj", (I, D)), ("up_proj", (I, D)), ("down_proj", (D, I))):
            w = torch.randint(0, 256, (epr, n, k // 2), dtype=torch.uint8, device=dev, generator=gl)
            s = torch.randint(120, 129, (epr, n, k // 32), dtype=torch.uint8, device=dev,
                              generator=gl)
            out[name] = (w, s)
        return out

    @classmethod
    def random_init(cls, q, torch, dev, rank, world, E, D, I, topk, seed=0):
        """Random weights of the release layout; the router and shared expert are the
        same on every rank (same seed), each rank draws only its own experts."""
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        epr = E // world
        m, g = cls._random_layer(q, torch, dev, epr, D, I, topk, seed)
        gate_w, gate_b = cls._draw_replicated(torch, dev, m, g, E, D, I)
        # the local layer's own router is not used (routing is over all E experts)
        m.gate.weight = gate_w[rank * epr:(rank + 1) * epr].contiguous()
        m.gate.bias = gate_b[rank * epr:(rank + 1) * epr].contiguous()
        for name, (w, s) in cls._draw_shard(torch, dev, rank, epr, D, I, seed).items():
            pr = getattr(m.experts, name)
            pr.weight, pr.scales = w, s
        ep = cls(m, world, rank, E)
        ep.gate_w, ep.gate_b = gate_w, gate_b
        ep.topk = topk
        return ep

    @classmethod
    def random_init_full(cls, q, torch, dev, world, E, D, I, topk, seed=0):
        """The single-GPU layer holding what ``random_init`` gives the ``world`` ranks
        together: the same router and shared expert, every rank's experts in rank order
        (a single-GPU reference for the sharded layer)."""
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        epr = E // world
        m, g = cls._random_layer(q, torch, dev, E, D, I, topk, seed)
        m.gate.weight, m.gate.bias = cls._draw_replicated(torch, dev, m, g, E, D, I)
        parts = {"gate_proj": [], "up_proj": [], "down_proj": []}
        for r in range(world):
            for name, ws in cls._draw_shard(torch, dev, r, epr, D, I, seed).items():
                parts[name].append(ws)
        for name, lst in parts.items():
            pr = getattr(m.experts, name)
            pr.weight = torch.cat([w for w, _ in lst])
            pr.scales = torch.cat([s for _, s in lst])
            lst.clear()
        return m

    def route(self, xf):
        """Replicated router over all E experts (moe.py:58-74)."""
        t = L.torch()
        T, D = xf.shape
        k = self.topk
        w = t.empty((T, k), dtype=t.float32, device=xf.device)
        idx = t.empty((T, k), dtype=t.int32, device=xf.device)
        ws = L.workspace(L.load().dsv41_moe_route_workspace_size(T, D, self.E), xf.device)
        L.call("dsv41_moe_route", L.ptr(xf), T, D, L.ptr(self.gate_w), L.ptr(self.gate_b), self.E, k,
               0, 1.0, 1, 1.5, L.ptr(w), L.ptr(idx), L.ptr(ws), ws.numel(), L.stream_of(xf))
        return w, idx

    def full_routing(self, x):
        xf = x.reshape(-1, x.shape[-1]).to(L.torch().bfloat16)
        w, idx = self.route(xf)
        return None, w, idx

    @property
    def local_active_mean(self):
        return sum(self.local_active) / max(len(self.local_active), 1)

    def _local_experts(self, rows, local_ids):
        """Owner side: each received row is one pair -> fp32 [R, D] via dsv41_moe_experts."""
        t = L.torch()
        m = self.local
        R = rows.shape[0]
        if R == 0:
            return t.empty((0, m.dim), dtype=t.float32, device=rows.device)
        cfg, W = m._decode_args(L.MOE_NO_SHARED)      # decode-packed scales when they apply
        cfg.topk = 1                                   # every received row is one pair
        y = t.empty((R, 1, m.dim), dtype=t.float32, device=rows.device)
        ws = L.workspace(L.load().dsv41_moe_decode_workspace_size(C.byref(cfg), R), rows.device)
        ids = local_ids.reshape(R, 1).contiguous()
        L.call("dsv41_moe_experts", C.byref(cfg), C.byref(W), L.ptr(rows), R, L.ptr(ids), L.ptr(y),
               L.ptr(ws), ws.numel(), L.stream_of(rows))
        return y[:, 0]

    def _shared(self, xf):
        """Shared expert on this rank's tokens (port numerics: bf16 intermediates)."""
        t = L.torch()
        from .linear import linear_fp8
        s = self.local.shared_experts
        g = linear_fp8(xf, s.w1.weight, s.w1.scales).float()
        u = linear_fp8(xf, s.w3.weight, s.w3.scales).float()
        lim = s.limit
        u = t.clamp(u, -lim, lim)
        g = t.clamp(g, max=lim)
        h = (t.nn.functional.silu(g) * u).to(t.bfloat16)
        return linear_fp8(h, s.w2.weight, s.w2.scales, out_dtype=t.bfloat16).float()

    # ---------------------------------------------------------------- prefill (a8)
    def forward_prefill(self, x, weights=None, indices=None, out_dtype=None):
        """The MoE layer at prefill (a8 numerics) with experts sharded over the group.  Each
        pair travels once as a packed fp8 row (codes, ue8m0 scales, owner-local expert,
        routing weight); owners run the grouped GEMMs and return bf16 rows; the source sums
        them per token in ascending expert order and adds the shared expert, which runs on
        a side stream during the exchange -- the same fp32 operations as one GPU."""
        t = L.torch()
        lib = L.load()
        xf = x.reshape(-1, x.shape[-1]).to(t.bfloat16).contiguous()
        T, D = xf.shape
        k = self.topk
        if indices is None:
            w, idx = self.route(xf)
        else:
            w, idx = weights.float().contiguous(), indices.to(t.int32).contiguous()
        dev = xf.device
        main = t.cuda.current_stream(dev)
        m = self.local
        lcfg = m._cfg(L.MOE_NO_SHARED)
        lcfg.topk = 1
        W = m._weights()
        packed = m._packed_scales(lcfg, W, dev)   # (re)packed on this stream, before the fork
        # shared expert on its own stream, overlapping the exchange and the routed experts
        if not hasattr(self, "_side"):
            self._side = t.cuda.Stream(device=dev)
        self._side.wait_stream(main)
        with t.cuda.stream(self._side):
            sh = m.prefill_a8(xf, out_dtype=t.bfloat16, routed=False)
        # pack the pairs by owner
        gcfg = m._cfg(L.MOE_NO_SHARED)
        gcfg.n_experts = self.E
        gcfg.topk = k
        P = T * k
        rb = lib.dsv41_moe_ep_row_bytes(D)
        send = t.empty((P, rb), dtype=t.uint8, device=dev)
        counts = t.empty((self.world,), dtype=t.int64, device=dev)
        slot_pos = t.empty((P,), dtype=t.int32, device=dev)
        ws = L.workspace(lib.dsv41_moe_ep_pack_workspace_size(C.byref(gcfg), T), dev)
        L.call("dsv41_moe_ep_pack", C.byref(gcfg), L.ptr(xf), T, L.ptr(w), L.ptr(idx),
               self.world, L.ptr(send), L.ptr(counts), L.ptr(slot_pos), L.ptr(ws), ws.numel(),
               L.stream_of(xf))
        recv_counts = exchange_counts(self.dist, counts, self.group)
        sc, rc = counts.tolist(), recv_counts.tolist()
        R = int(sum(rc))
        recv = t.empty((R, rb), dtype=t.uint8, device=dev)
        self.dist.all_to_all_single(recv, send, rc, sc, group=self.group)
        # owner: this rank's experts on the received rows
        y_recv = t.empty((R, D), dtype=t.bfloat16, device=dev)
        if R:
            ws2 = L.workspace(lib.dsv41_moe_ep_experts_workspace_size(C.byref(lcfg), R, 1), dev)
            L.call("dsv41_moe_ep_experts", C.byref(lcfg), C.byref(W), L.ptr(packed), L.ptr(recv),
                   R, L.ptr(y_recv), L.ptr(ws2), ws2.numel(), L.stream_of(xf))
        if self.track:
            self.local_active.append(R)
        back = t.empty((P, D), dtype=t.bfloat16, device=dev)
        self.dist.all_to_all_single(back, y_recv, sc, rc, group=self.group)
        main.wait_stream(self._side)
        sh.record_stream(main)
        odt = out_dtype or (t.float32 if x.dtype == t.float32 else t.bfloat16)
        out = t.empty((T, D), dtype=odt, device=dev)
        L.call("dsv41_moe_ep_combine", L.ptr(back), L.ptr(slot_pos), L.ptr(idx), L.ptr(sh), T, k,
               D, L.dtype_code(odt), L.ptr(out), L.stream_of(xf))
        return out.reshape(tuple(x.shape[:-1]) + (D,))

    # ---------------------------------------------------------------- decode over peer memory
    def _ensure_ctx(self, dev):
        """This rank's exchange buffer, with every peer's buffer mapped (collective: every rank
        calls it once, on the first decode step)."""
        if self._ctx is not None:
            return self._ctx
        t = L.torch()
        lib = L.load()
        ctx = C.c_void_p()
        L.call("dsv41_ep_create", self.world, self.rank, self.max_tokens, self.topk,
               self.local.dim, C.byref(ctx))
        nb = int(lib.dsv41_ep_handle_bytes())
        h = (C.c_uint8 * nb)()
        L.call("dsv41_ep_handle", ctx, C.cast(h, C.c_void_p))
        mine = t.tensor(list(bytes(h)), dtype=t.uint8, device=dev)
        every = t.empty(nb * self.world, dtype=t.uint8, device=dev)
        self.dist.all_gather_into_tensor(every, mine, group=self.group)
        hb = (C.c_uint8 * (nb * self.world)).from_buffer_copy(bytes(every.cpu().numpy().tobytes()))
        L.call("dsv41_ep_connect", ctx, C.cast(hb, C.c_void_p))
        self.dist.barrier(group=self.group)            # every peer mapped before any step
        self._ctx = ctx
        return ctx

    def close(self):
        """Unmap the peers and free the exchange buffer (collective)."""
        if self._ctx is not None:
            L.torch().cuda.synchronize()
            self.dist.barrier(group=self.group)
            L.call("dsv41_ep_destroy", self._ctx)
            self._ctx = None

    def _forward_p2p(self, xf, odt):
        """One decode step: dsv41_moe_ep_decode (pairs to their owners and back through
        NVLink peer stores, no host synchronisation)."""
        t = L.torch()
        lib = L.load()
        T, D = xf.shape
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the EP buffers")
        ctx = self._ensure_ctx(xf.device)
        m = self.local
        cfg, W = m._decode_args()                      # shared + this rank's experts
        cfg.n_experts = self.E
        W.gate_w, W.gate_bias = L.ptr(self.gate_w), L.ptr(self.gate_b)
        need = int(lib.dsv41_moe_ep_decode_workspace_size(C.byref(cfg), ctx, T))
        if self._ws is None or self._ws.numel() < need or self._ws.device != xf.device:
            self._ws = L.workspace(need, xf.device)
        k = self.topk
        y = t.empty((T, D), dtype=odt, device=xf.device)
        w = t.empty((T, k), dtype=t.float32, device=xf.device)
        idx = t.empty((T, k), dtype=t.int32, device=xf.device)
        L.call("dsv41_moe_ep_decode", C.byref(cfg), C.byref(W), ctx, L.ptr(xf) if T else None, T,
               L.dtype_code(odt), L.ptr(y) if T else None, L.ptr(w) if T else None,
               L.ptr(idx) if T else None, L.ptr(self._ws), self._ws.numel(), L.stream_of(xf))
        return y, w, idx

    def forward(self, x, expert_fn=None, with_routing=False):
        t = L.torch()
        xf = x.reshape(-1, x.shape[-1]).to(t.bfloat16).contiguous()
        T = xf.shape[0]
        if expert_fn is None and not self.track and self.p2p and xf.is_cuda:
            odt = t.float32 if x.dtype == t.float32 else t.bfloat16
            y, w, idx = self._forward_p2p(xf, odt)
            out = y.reshape(x.shape)
            return (out, w, idx) if with_routing else out
        w, idx = self.route(xf)
        rows, ids, order, sc, rc = dispatch(self.dist, xf, idx, self.world, self.epr, self.group)
        if self.track:
            self.local_active.append(int(t.unique(ids).numel()))
        fn = expert_fn or self._local_experts
        y_recv = fn(rows, ids)
        Y = combine(self.dist, y_recv, order, sc, rc, T, self.topk, self.group)
        out = weighted_sum(Y, w, self._shared(xf)).to(x.dtype if x.dtype != t.float32 else t.float32)
        out = out.reshape(x.shape)
        return (out, w, idx) if with_routing else out
