"""Expert parallelism for the MoE layer (training and rollout).

Each rank of the expert-parallel group owns E / ep consecutive experts. For a batch of local
tokens:

  1. route (replicated router on local tokens; or R3-replayed routing)
  2. plan the send order with the deterministic permute kernel, using destination ranks as the
     groups (entries (t, j) ordered by destination rank, then token, then slot)
  3. exchange row counts, then all-to-all the hidden rows and their local expert ids
  4. received rows -> expert-sorted 128-row padded segments -> grouped tcgen05 GEMMs
  5. reverse all-to-all of the expert outputs, then the fixed-order weighted combine
The backward runs the same exchanges in reverse. Two transports: NCCL all-to-all
(`all_to_all_single`, steps 3 and 5 above), and in-kernel peer memory (`_MoEEPPeer`,
csrc/moe_ep.cu): the dispatch kernel stores every row straight into its owner's expert-sorted
buffer and the combine kernel loads the expert outputs from the owners, with device barriers
instead of host synchronisation. Either way the order of every row is a pure function of
(source rank, token, slot), so results do not depend on timing, and both equal the single-GPU
layer bit for bit. On CPU ranks (gloo) `moe_ep_ref` runs the same exchange in PyTorch autograd.

Under TP the experts are either split over the TP ranks as well (expert-tensor parallel size =
TP; the EP group is the ranks with the same TP rank) or whole (size 1; each TP rank routes its
share of the replicated rows): `Transformer._routed`.

Reference: Megatron MoE alltoall token dispatcher (--moe-token-dispatcher-type alltoall),
DeepEP flex dispatcher (--moe-enable-deepep), expert index offsets for naming
(update_weight/common.py:186-190), --expert-tensor-parallel-size (utils/arguments.py).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from miles_b200.ops import gemm as G
from miles_b200.ops._lib import lib
from miles_b200.ops.moe import ALIGN, MoEPlan, RouterCfg, _accum_grouped_wgrad, emit_record, router_bias


class EPContext:
    def __init__(self, group, num_experts: int, transport: str = "auto", hidden: int = 0,
                 topk: int = 8, cap_tokens: int = 16384):
        """transport "peer": dispatch / combine by kernels storing into and loading from the
        other ranks' symmetric buffers (csrc/moe_ep.cu); "nccl": all-to-all collectives;
        "auto": peer under NCCL (one node), else the collectives."""
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        assert num_experts % self.size == 0
        self.E = num_experts
        self.E_local = num_experts // self.size
        self.first = self.rank * self.E_local
        if transport == "auto":
            transport = "peer" if dist.get_backend(group) == "nccl" and hidden > 0 else "nccl"
        self.transport = transport
        self.hidden, self.topk, self.cap_tokens = hidden, topk, cap_tokens
        self._peer = None

    def peer(self):
        if self._peer is None:
            self._peer = EPPeerBuffers(self)
        return self._peer


class EPPeerBuffers:
    """Symmetric region of one EP rank: flags | table [world][E_local] | base [E_local][world] |
    xs [cap][H] | ys [cap][H] (cap = world * cap_tokens * k rows + 128-row padding per expert)."""

    def __init__(self, ep: "EPContext"):
        from miles_b200.ops._lib import err_word
        from miles_b200.parallel.symm import SymmBuffer

        W, El, H = ep.size, ep.E_local, ep.hidden
        self.cap = W * ep.cap_tokens * ep.topk + El * ALIGN
        self.t_off = 256
        self.b_off = self.t_off + ((W * El * 4 + 255) // 256) * 256
        self.x_off = self.b_off + ((El * W * 4 + 255) // 256) * 256
        self.y_off = self.x_off + self.cap * H * 2
        dev = torch.device("cuda", torch.cuda.current_device())
        self.buf = SymmBuffer(self.y_off + self.cap * H * 2, ep.group, dev)
        P = self.buf.peers
        self.flag_ptrs = list(P)
        self.table_ptrs = [p + self.t_off for p in P]
        self.base_ptrs = [p + self.b_off for p in P]
        self.xs_ptrs = [p + self.x_off for p in P]
        self.ys_ptrs = [p + self.y_off for p in P]
        self.my_flags = self.buf.view(0, (8,), torch.int32)
        self.table = self.buf.view(self.t_off, (W * El,), torch.int32)
        self.base = self.buf.view(self.b_off, (El * W,), torch.int32)
        self.xs = self.buf.view(self.x_off, (self.cap, H), torch.bfloat16)
        self.ys = self.buf.view(self.y_off, (self.cap, H), torch.bfloat16)
        self.ctl = torch.zeros(4, dtype=torch.int32, device=dev)
        self.err = err_word(dev)
        self.ep = ep

    def barrier(self):
        lib().symm_barrier(self.flag_ptrs, self.my_flags, self.ctl, self.ep.rank, self.ep.size,
                           2_000_000_000, self.err)


class _RecvPlan:
    """Grouped-GEMM plan of the rows an owner received (device offsets / counts, host bounds)."""

    def __init__(self, offsets, counts, E, rows, n_rows):
        self.offsets, self.counts, self.E, self.rows = offsets, counts, E, rows
        self.T, self.k = n_rows, 1

    @property
    def total_rows(self):
        return self.offsets[self.E:]


class _MoEEPPeer(torch.autograd.Function):
    """Expert-parallel MoE layer with in-kernel dispatch / combine over peer memory (see
    csrc/moe_ep.cu for the steps and their ordering)."""

    @staticmethod
    def forward(ctx, x, router_w, w1, w2, bias, cfg: RouterCfg, ep: EPContext, replay_idx, record,
                need_bwd):
        T, H = x.shape
        k = cfg.k
        x = x.contiguous()
        B = ep.peer()
        C = lib()
        dev = x.device
        logits = G.matmul_nt(x, router_w, out_dtype=torch.float32)
        idx = torch.empty(T, k, dtype=torch.int32, device=dev)
        w = torch.empty(T, k, dtype=torch.float32, device=dev)
        C.router_fwd(logits, router_bias(bias), replay_idx, idx, w, k, cfg.score_fn, cfg.renorm,
                     cfg.n_group, cfg.topk_group, cfg.scale)
        emit_record(record, idx)
        if T > ep.cap_tokens:
            raise ValueError(f"{T} tokens exceed the EP buffers ({ep.cap_tokens})")
        n = T * k
        nch = max(1, (n + 1023) // 1024)
        hist = torch.empty(nch * ep.E, dtype=torch.int32, device=dev)
        hbase = torch.empty_like(hist)
        counts_g = torch.empty(ep.E, dtype=torch.int32, device=dev)
        off_g = torch.empty(ep.E + 1, dtype=torch.int32, device=dev)
        dest_g = torch.empty(n, dtype=torch.int32, device=dev)
        C.moe_permute_plan(idx.view(-1), ep.E, 1, hist, hbase, counts_g, off_g, dest_g)
        C.ep_publish(counts_g, ep.E_local, ep.rank, B.table_ptrs)
        B.barrier()
        offsets = torch.empty(ep.E_local + 1, dtype=torch.int32, device=dev)
        counts = torch.empty(ep.E_local, dtype=torch.int32, device=dev)
        C.ep_offsets(B.table, ep.size, ep.E_local, ALIGN, offsets, counts, B.base, B.cap, B.err)
        B.barrier()
        pos = torch.empty(n, dtype=torch.int32, device=dev)
        C.ep_dispatch(x, idx, dest_g, off_g, ep.E_local, ep.rank, B.base_ptrs, B.xs_ptrs, B.cap, pos, B.err)
        B.barrier()
        # owner: grouped expert GEMMs on the received rows
        nb = ep.size * T * k  # bound on received rows (ranks run equal micro-batch shapes)
        plan = _RecvPlan(offsets, counts, ep.E_local, B.cap, nb)
        if need_bwd:
            xs = B.xs.clone()
            C.moe_zero_pad(counts, offsets, xs)
        else:
            xs = B.xs
        cnt = None if need_bwd else counts
        a, gu = G.grouped_nt_swiglu(xs, w1, offsets, n_rows=nb, save_gu=need_bwd, counts=cnt)
        G.grouped_nt(a, w2, offsets, out=B.ys, n_rows=nb, counts=cnt)
        B.barrier()
        y = torch.empty_like(x)
        saved = torch.empty(n, H, dtype=x.dtype, device=dev) if need_bwd else None
        C.ep_combine(B.ys_ptrs, idx, pos, w, None, H, ep.E_local, y, saved)
        if need_bwd:
            ctx.save_for_backward(x, router_w, w1, w2, logits, idx, w, pos, xs, gu, a, saved,
                                  offsets, counts)
            ctx.misc = (cfg, ep, plan)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, router_w, w1, w2, logits, idx, w, pos, xs, gu, a, saved, offsets, counts = ctx.saved_tensors
        cfg, ep, plan = ctx.misc
        B = ep.peer()
        C = lib()
        T, H = x.shape
        dy = dy.contiguous()
        B.barrier()  # every rank is done reading the ys buffers of the forward combine
        dw = torch.empty_like(w)
        C.ep_combine_bwd(dy, saved, idx, pos, w, ep.E_local, B.ys_ptrs, dw)
        B.barrier()
        dys = B.ys
        C.moe_zero_pad(counts, offsets, dys)
        da = G.grouped_nn(dys, w2, offsets)
        dw2 = _accum_grouped_wgrad(w2, dys, a, plan)
        dgu = torch.empty_like(gu)
        C.swiglu_bwd(gu, da, dgu, plan.total_rows)
        G.grouped_nn(dgu, w1, offsets, out=B.xs)
        dw1 = _accum_grouped_wgrad(w1, dgu, xs, plan)
        B.barrier()
        dx = torch.empty_like(x)
        C.ep_gather_bwd(B.xs_ptrs, idx, pos, H, ep.E_local, dx)
        dlogits = torch.empty(T, cfg.E, dtype=torch.bfloat16, device=x.device)
        C.router_bwd(logits, idx, dw, dlogits, cfg.score_fn, cfg.renorm, cfg.scale)
        dx.add_(G.matmul_nn(dlogits, router_w))
        dwr = G._accumulate_wgrad(router_w, dlogits, x)
        return dx, dwr, dw1, dw2, None, None, None, None, None, None


def _exchange_counts(send_counts: torch.Tensor, ep: EPContext) -> torch.Tensor:
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts, group=ep.group)
    return recv


def _a2a(x: torch.Tensor, send_splits: list[int], recv_splits: list[int], ep: EPContext):
    out = x.new_empty((sum(recv_splits),) + tuple(x.shape[1:]))
    dist.all_to_all_single(out, x.contiguous(), recv_splits, send_splits, group=ep.group)
    return out


class _MoEEP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, router_w, w1, w2, bias, cfg: RouterCfg, ep: EPContext, replay_idx, record,
                need_bwd):
        T, H = x.shape
        k = cfg.k
        x = x.contiguous()
        logits = G.matmul_nt(x, router_w, out_dtype=torch.float32)
        idx = torch.empty(T, k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, k, dtype=torch.float32, device=x.device)
        lib().router_fwd(logits, router_bias(bias), replay_idx, idx, w, k, cfg.score_fn, cfg.renorm,
                         cfg.n_group, cfg.topk_group, cfg.scale)
        emit_record(record, idx)
        # send plan: groups = destination ranks, no padding
        dest_rank = torch.div(idx, ep.E_local, rounding_mode="floor").to(torch.int32)
        n = T * k
        nch = max(1, (n + 1023) // 1024)
        hist = torch.empty(nch * ep.size, dtype=torch.int32, device=x.device)
        base = torch.empty_like(hist)
        send_counts = torch.empty(ep.size, dtype=torch.int32, device=x.device)
        send_off = torch.empty(ep.size + 1, dtype=torch.int32, device=x.device)
        send_pos = torch.empty(n, dtype=torch.int32, device=x.device)
        lib().moe_permute_plan(dest_rank.view(-1), ep.size, 1, hist, base, send_counts, send_off, send_pos)
        send_x = torch.empty(n, H, dtype=x.dtype, device=x.device)
        lib().moe_gather(x, send_pos, k, send_x)
        local_eid = (idx - dest_rank * ep.E_local).view(-1)
        send_eid = torch.empty(n, dtype=torch.int32, device=x.device)
        send_eid.index_copy_(0, send_pos.long(), local_eid.to(torch.int32))
        recv_counts = _exchange_counts(send_counts, ep)
        ss, rs = send_counts.tolist(), recv_counts.tolist()
        recv_x = _a2a(send_x, ss, rs, ep)
        recv_eid = _a2a(send_eid, ss, rs, ep)
        # local experts on the received rows (one "token" per row, k = 1)
        plan = MoEPlan(recv_eid.view(-1, 1), ep.E_local)
        xs = plan.gather(recv_x, zero_pad=need_bwd)
        gu = G.grouped_nt(xs, w1, plan.offsets)
        a = torch.empty(gu.shape[0], gu.shape[1] // 2, dtype=gu.dtype, device=gu.device)
        lib().swiglu_fwd(gu, a, plan.total_rows)
        ys = G.grouped_nt(a, w2, plan.offsets)
        back = torch.empty(recv_x.shape[0], H, dtype=x.dtype, device=x.device)
        if back.shape[0]:
            ones = torch.ones(back.shape[0], 1, dtype=torch.float32, device=x.device)
            lib().moe_combine(ys, plan.dest, ones, None, back)
        ret = _a2a(back, rs, ss, ep)  # rows back in send order
        y = torch.empty_like(x)
        lib().moe_combine(ret, send_pos, w, None, y)
        ctx.save_for_backward(x, router_w, w1, w2, logits, idx, w, send_pos, xs, gu, a, ret)
        ctx.misc = (cfg, ep, plan, ss, rs)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, router_w, w1, w2, logits, idx, w, send_pos, xs, gu, a, ret = ctx.saved_tensors
        cfg, ep, plan, ss, rs = ctx.misc
        T, H = x.shape
        k = cfg.k
        dy = dy.contiguous()
        dret = torch.empty_like(ret)
        dw = torch.empty_like(w)
        lib().moe_combine_bwd(dy, ret, send_pos, w, dret, dw)
        dback = _a2a(dret, ss, rs, ep)                    # gradient w.r.t. `back`
        dys = torch.empty(plan.rows, H, dtype=x.dtype, device=x.device)
        lib().moe_gather(dback, plan.dest, 1, dys)        # back[r] = ys[dest[r]] -> scatter
        lib().moe_zero_pad(plan.counts, plan.offsets, dys)
        da = G.grouped_nn(dys, w2, plan.offsets)
        dw2 = _accum_grouped_wgrad(w2, dys, a, plan)
        dgu = torch.empty_like(gu)
        lib().swiglu_bwd(gu, da, dgu, plan.total_rows)
        dxs = G.grouped_nn(dgu, w1, plan.offsets)
        dw1 = _accum_grouped_wgrad(w1, dgu, xs, plan)
        drecv = torch.empty(dback.shape[0], H, dtype=x.dtype, device=x.device)
        if drecv.shape[0]:
            lib().moe_gather_bwd(dxs, plan.dest, 1, drecv)
        dsend = _a2a(drecv, rs, ss, ep)
        dx = torch.empty_like(x)
        lib().moe_gather_bwd(dsend, send_pos, k, dx)
        dlogits = torch.empty(T, cfg.E, dtype=torch.bfloat16, device=x.device)
        lib().router_bwd(logits, idx, dw, dlogits, cfg.score_fn, cfg.renorm, cfg.scale)
        dx.add_(G.matmul_nn(dlogits, router_w))
        dwr = G._accumulate_wgrad(router_w, dlogits, x)
        return dx, dwr, dw1, dw2, None, None, None, None, None, None


class _A2A(torch.autograd.Function):
    """Differentiable all-to-all of rows: the backward sends the gradients the reverse way."""

    @staticmethod
    def forward(ctx, x, send_splits, recv_splits, ep):
        ctx.misc = (send_splits, recv_splits, ep)
        return _a2a(x, send_splits, recv_splits, ep)

    @staticmethod
    def backward(ctx, g):
        ss, rs, ep = ctx.misc
        return _a2a(g, rs, ss, ep), None, None, None


def moe_ep_ref(x, router_w, w1_local, w2_local, cfg: RouterCfg, ep: EPContext, bias=None,
               replay_idx=None, record=None):
    """PyTorch expert-parallel layer (CPU ranks, gloo): the same exchange as the kernel path
    (rows ordered by destination rank, then token, then slot; counts, rows and local expert
    ids all-to-all; reverse all-to-all of the expert outputs; weighted combine) in autograd
    ops, experts in fp32. Equals `moe_ref` over the global expert set."""
    from miles_b200.ops.moe import route_ref, swiglu_ref

    T, H = x.shape
    logits = x.float() @ router_w.float().t()
    idx, w = route_ref(logits, cfg, bias, replay_idx)
    emit_record(record, idx)
    dest = torch.div(idx.long(), ep.E_local, rounding_mode="floor").view(-1)
    # stable sort by destination keeps (token, slot) order inside each destination
    order = torch.sort(dest, stable=True).indices
    tok = torch.div(order, cfg.k, rounding_mode="floor")
    send_counts = torch.bincount(dest, minlength=ep.size).to(torch.int64)
    recv_counts = _exchange_counts(send_counts, ep)
    ss, rs = send_counts.tolist(), recv_counts.tolist()
    send_eid = (idx.long().view(-1) - dest * ep.E_local)[order]
    recv_x = _A2A.apply(x[tok].float(), ss, rs, ep)
    recv_eid = _a2a(send_eid, ss, rs, ep)
    rd = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
    out = torch.zeros(recv_x.shape[0], H, dtype=torch.float32, device=x.device)
    for e in range(ep.E_local):
        rows = (recv_eid == e).nonzero(as_tuple=True)[0]
        if rows.numel() == 0:
            continue
        gu = (recv_x[rows] @ w1_local[e].float().t()).to(rd)
        o = (swiglu_ref(gu).float() @ w2_local[e].float().t()).to(rd)
        out = out.index_add(0, rows, o.float())
    ret = _A2A.apply(out, rs, ss, ep)
    wf = w.view(-1)[order]
    y = torch.zeros(T, H, dtype=torch.float32, device=x.device).index_add(0, tok, wf[:, None] * ret)
    return y.to(x.dtype)


def moe_experts_ep(x, router_w, w1_local, w2_local, cfg: RouterCfg, ep: EPContext, bias=None,
                   replay_idx=None, record=None):
    """Expert-parallel MoE: w1_local [E/ep, 2I, H], w2_local [E/ep, H, I] hold this rank's
    experts; routing and the output are over the global expert set."""
    from miles_b200.ops._lib import use_native

    if not use_native(x):
        return moe_ep_ref(x, router_w, w1_local, w2_local, cfg, ep, bias, replay_idx, record)
    fn = _MoEEPPeer if (ep.transport == "peer" and x.is_cuda) else _MoEEP
    return fn.apply(x, router_w, w1_local, w2_local, bias, cfg, ep, replay_idx, record,
                    torch.is_grad_enabled())
