"""Mixture-of-experts layer on the sm_100a kernels (csrc/moe.cu + grouped tcgen05 GEMMs).

    logits = x @ Wr^T (fp32)            router_fwd  -> top-k experts / weights (or R3 replay)
    plan: deterministic expert-sorted order, 128-row padded segments
    xs = gather(x); gu = xs @ W1[e]^T; a = swiglu(gu); ys = a @ W2[e]^T; y = sum_j w_j ys

The backward mirrors it with grouped data-grad (K, MN-major) and weight-grad (MN, MN-major)
GEMMs; every reduction is fixed-order, so the layer is bitwise reproducible.

Reference roles replaced: Megatron MoE layer with TEGroupedLinear and alltoall dispatcher,
router with R3 replay (megatron.patch:514-541), fsdp_utils/kernels/fused_experts.py.
"""
from __future__ import annotations

import torch

from miles_b200.ops import gemm as G
from miles_b200.ops._lib import lib, use_native
from miles_b200.ops.norm import swiglu_ref

FUSED_DISPATCH_MAX_ROWS = 4096  # T * k limit of the fused route + dispatch kernel
ALIGN = 128


class RouterCfg:
    def __init__(self, num_experts: int, topk: int, score_fn: str = "softmax", renorm: bool = True,
                 n_group: int = 1, topk_group: int = 1, scale: float = 1.0):
        self.E = num_experts
        self.k = topk
        self.score_fn = 0 if score_fn == "softmax" else 1
        self.renorm = renorm
        self.n_group = n_group
        self.topk_group = topk_group
        self.scale = scale


def route_ref(logits: torch.Tensor, cfg: RouterCfg, bias=None, replay_idx=None):
    """fp32 reference router: returns (idx int32 [T,k], weights fp32 [T,k])."""
    if cfg.score_fn == 0:
        sc = logits.float().softmax(-1)
        sel = sc
    else:
        sc = logits.float().sigmoid()
        sel = sc + (bias.float() if bias is not None else 0)
        if cfg.n_group > 1:
            T = sel.shape[0]
            g = sel.view(T, cfg.n_group, -1)
            gs = g.topk(2, -1).values.sum(-1)
            keep = gs.topk(cfg.topk_group, -1).indices
            mask = torch.zeros_like(gs, dtype=torch.bool).scatter_(1, keep, True)
            sel = sel.masked_fill(~mask.repeat_interleave(g.shape[-1], 1), float("-inf"))
    if replay_idx is not None:
        idx = replay_idx.long()
    else:
        idx = torch.sort(sel, dim=-1, descending=True, stable=True).indices[:, : cfg.k]
    w = sc.gather(1, idx)
    if cfg.renorm:
        w = w / w.sum(-1, keepdim=True)
    return idx.int(), (w * cfg.scale).float()


def moe_ref(x, router_w, w1, w2, cfg: RouterCfg, bias=None, replay_idx=None):
    """fp32 reference of the whole expert layer."""
    from miles_b200.ops.fp8 import fp8_of, quant_act_ref

    logits = x.float() @ router_w.float().t()
    idx, w = route_ref(logits, cfg, bias, replay_idx)
    T, H = x.shape
    w1q, w2q = fp8_of(w1), fp8_of(w2)
    if w1q is not None and w2q is not None:
        # block-scaled fp8 experts: quantise-dequantise both operands of each expert GEMM
        # (the fp8 values in the forward; gradients pass straight through to the bf16 operands)
        def qdq(a):
            q, s = quant_act_ref(a.detach())
            K = a.shape[1]
            return a + ((q.float().view(-1, K // 128, 128) * s.t()[..., None]).view(-1, K) - a).detach()

        w1 = w1 + (w1q.dequant().view(w1.shape) - w1).detach()
        w2 = w2 + (w2q.dequant().view(w2.shape) - w2).detach()
    else:
        def qdq(a):
            return a
    y = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for e in range(cfg.E):
        tok, slot = (idx == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        # intermediate roundings follow the activation dtype (bf16 on the kernel path)
        rd = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float32
        gu = (qdq(x[tok].float()) @ w1[e].float().t()).to(rd)
        a = swiglu_ref(gu)
        o = (qdq(a.float()) @ w2[e].float().t()).to(rd)
        y.index_add_(0, tok, w[tok, slot][:, None] * o.float())
    return y.to(x.dtype), idx


class MoEPlan:
    """Device-side dispatch plan for one batch: dest rows, padded offsets and counts."""

    @classmethod
    def fused(cls, logits, bias, replay_idx, x, cfg: "RouterCfg", idx_out=None):
        """Routing + plan + gather in one kernel (small batches, no backward). Returns
        (plan, idx, w, xs); idx_out: optional contiguous int32 [T, k] that receives idx."""
        T = logits.shape[0]
        k, E = cfg.k, cfg.E
        n = T * k
        dev = logits.device
        self = cls.__new__(cls)
        self.E, self.k, self.T = E, k, T
        self.rows = ((n + E * (ALIGN - 1)) + ALIGN - 1) // ALIGN * ALIGN
        self.counts = torch.empty(E, dtype=torch.int32, device=dev)
        self.offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        self.dest = torch.empty(n, dtype=torch.int32, device=dev)
        idx = idx_out if idx_out is not None else torch.empty(T, k, dtype=torch.int32, device=dev)
        w = torch.empty(T, k, dtype=torch.float32, device=dev)
        xs = torch.empty(self.rows, x.shape[1], dtype=x.dtype, device=dev)
        lib().moe_route_dispatch(logits, bias, replay_idx, x, idx, w, self.counts, self.offsets,
                                 self.dest, xs, k, cfg.score_fn, cfg.renorm, cfg.n_group,
                                 cfg.topk_group, cfg.scale, ALIGN)
        return self, idx, w, xs

    def __init__(self, idx: torch.Tensor, E: int):
        T, k = idx.shape
        n = T * k
        dev = idx.device
        nchunks = max(1, (n + 1023) // 1024)
        self.E, self.k, self.T = E, k, T
        self.rows = ((n + E * (ALIGN - 1)) + ALIGN - 1) // ALIGN * ALIGN
        hist = torch.empty(nchunks * E, dtype=torch.int32, device=dev)
        base = torch.empty(nchunks * E, dtype=torch.int32, device=dev)
        self.counts = torch.empty(E, dtype=torch.int32, device=dev)
        self.offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        self.dest = torch.empty(n, dtype=torch.int32, device=dev)
        lib().moe_permute_plan(idx.contiguous().view(-1), E, ALIGN, hist, base, self.counts,
                               self.offsets, self.dest)

    def gather(self, x: torch.Tensor, zero_pad: bool = True) -> torch.Tensor:
        """Expert-sorted copy of x. Padding rows only matter to the weight-grad contraction, so
        they are zeroed only when a backward will follow."""
        xs = torch.empty(self.rows, x.shape[1], dtype=x.dtype, device=x.device)
        lib().moe_gather(x, self.dest, self.k, xs)
        if zero_pad:
            lib().moe_zero_pad(self.counts, self.offsets, xs)
        return xs

    @property
    def total_rows(self) -> torch.Tensor:
        return self.offsets[self.E:]


def _accum_grouped_wgrad(w: torch.Tensor, dy: torch.Tensor, x: torch.Tensor, plan: MoEPlan):
    main = G.main_grad_of(w)
    if main is not None:
        G.grouped_tn(dy, x, plan.offsets, plan.E, out=main, accumulate=True)
        return None
    return G.grouped_tn(dy, x, plan.offsets, plan.E)


def experts_forward(xs, w1, w2, plan: MoEPlan, save_gu: bool = True):
    """gate_up GEMM with the SwiGLU fused into its epilogue, then the down GEMM. The
    pre-activation gu is kept only when a backward follows."""
    from miles_b200.ops.fp8 import fp8_experts, fp8_of

    w1q, w2q = fp8_of(w1), fp8_of(w2)
    if w1q is not None and w2q is not None:
        E, N2, H = w1.shape
        return fp8_experts(xs, w1q, w2q, plan.offsets, plan.counts, E, N2 // 2, H, save_gu)
    n = plan.T * plan.k
    # without a backward the padding rows are never read: skip writing them
    cnt = None if save_gu else plan.counts
    a, gu = G.grouped_nt_swiglu(xs, w1, plan.offsets, n_rows=n, save_gu=save_gu, counts=cnt)
    ys = G.grouped_nt(a, w2, plan.offsets, n_rows=n, counts=cnt)
    return gu, a, ys


def router_bias(bias):
    """The routing-score bias as the fp32 vector the router kernels read (parameters may be
    stored in the model dtype)."""
    if bias is None or bias.dtype == torch.float32:
        return bias
    return bias.float().contiguous()


class _MoE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, router_w, w1, w2, bias, cfg: RouterCfg, replay_idx, record, need_bwd):
        T, H = x.shape
        bias = router_bias(bias)
        x = x.contiguous()
        logits = G.matmul_nt(x, router_w, out_dtype=torch.float32)
        if not need_bwd and T * cfg.k <= FUSED_DISPATCH_MAX_ROWS:
            # decode-sized batch: one kernel for routing, plan and gather
            into = record if isinstance(record, torch.Tensor) else None
            plan, idx, w, xs = MoEPlan.fused(logits, bias, replay_idx.contiguous().view(T, cfg.k)
                                             if replay_idx is not None else None, x, cfg, idx_out=into)
            if record is not None and into is None:
                record(idx)
        else:
            idx = torch.empty(T, cfg.k, dtype=torch.int32, device=x.device)
            w = torch.empty(T, cfg.k, dtype=torch.float32, device=x.device)
            lib().router_fwd(logits, bias, replay_idx, idx, w, cfg.k, cfg.score_fn, cfg.renorm,
                             cfg.n_group, cfg.topk_group, cfg.scale)
            emit_record(record, idx)
            plan = MoEPlan(idx, cfg.E)
            xs = plan.gather(x, zero_pad=need_bwd)
        gu, a, ys = experts_forward(xs, w1, w2, plan, save_gu=need_bwd)
        y = torch.empty_like(x)
        lib().moe_combine(ys, plan.dest, w, None, y)
        ctx.save_for_backward(x, router_w, w1, w2, logits, idx, w, xs, gu, a, ys)
        ctx.plan = plan
        ctx.cfg = cfg
        return y

    @staticmethod
    def backward(ctx, dy):
        x, router_w, w1, w2, logits, idx, w, xs, gu, a, ys = ctx.saved_tensors
        plan, cfg = ctx.plan, ctx.cfg
        dy = dy.contiguous()
        T, H = x.shape
        dys = torch.empty_like(ys)
        dw = torch.empty_like(w)
        lib().moe_combine_bwd(dy, ys, plan.dest, w, dys, dw)
        lib().moe_zero_pad(plan.counts, plan.offsets, dys)
        da = G.grouped_nn(dys, w2, plan.offsets)
        dw2 = _accum_grouped_wgrad(w2, dys, a, plan)
        dgu = torch.empty_like(gu)
        lib().swiglu_bwd(gu, da, dgu, plan.total_rows)
        dxs = G.grouped_nn(dgu, w1, plan.offsets)
        dw1 = _accum_grouped_wgrad(w1, dgu, xs, plan)
        dx = torch.empty_like(x)
        lib().moe_gather_bwd(dxs, plan.dest, plan.k, dx)
        dlogits = torch.empty(T, cfg.E, dtype=torch.bfloat16, device=x.device)
        lib().router_bwd(logits, idx, dw, dlogits, cfg.score_fn, cfg.renorm, cfg.scale)
        dx.add_(G.matmul_nn(dlogits, router_w))
        dwr = G._accumulate_wgrad(router_w, dlogits, x)
        return dx, dwr, dw1, dw2, None, None, None, None, None


def emit_record(record, idx: torch.Tensor) -> None:
    """Hand a layer's routing to its recorder: a callable, or an int32 [T, k] tensor that
    receives a copy (the decode path passes its record buffer so that the fused router kernel
    writes into it directly)."""
    if record is None:
        return
    if isinstance(record, torch.Tensor):
        if record.data_ptr() != idx.data_ptr():
            record.copy_(idx)
    else:
        record(idx)


def moe_experts(x, router_w, w1, w2, cfg: RouterCfg, bias=None, replay_idx=None, record=None):
    """Routed-expert output for x [T,H]. w1 [E, 2I, H] ([gate|up]), w2 [E, H, I].
    replay_idx: int32 [T,k] replays a recorded routing (R3); `record` receives the routing
    actually used (R3 capture): a callable record(idx) or an int32 [T, k] output tensor."""
    if not use_native(x):
        y, idx = moe_ref(x, router_w, w1, w2, cfg, bias, replay_idx)
        emit_record(record, idx)
        return y
    return _MoE.apply(x, router_w, w1, w2, bias, cfg, replay_idx, record, torch.is_grad_enabled())
