"""Tensor parallelism (Megatron-style column / row parallel layers) for the transformer.

Layout over a TP group of size t (rank r holds the r-th contiguous slice):
  * attention: query heads and KV heads are split t ways (qkv_proj rows, o_proj columns);
    MLA splits its heads the same way (q_proj / q_b_proj and kv_b_proj rows, o_proj columns),
    the latent projections (kv_a_proj_with_mqa, q_a_proj) stay replicated
  * dense MLP and shared experts: the intermediate dimension is split (gate_up rows, down
    columns); routed experts split their intermediate dimension the same way
  * embeddings, norms, the router and the LM head are replicated
A column-parallel projection takes `copy_to_tp(x)` (identity forward, all-reduce of the input
gradient backward); a row-parallel projection is followed by `reduce_from_tp` (all-reduce
forward, identity backward). Replicated parameters that only see this rank's heads or
intermediate slice (QK-norm weights; the router under a split MoE) get partial gradients,
which `tp_partial_param_names` lists and the trainer all-reduces over the TP group.

All-reduce backends:
  * "symm" (CUDA): the in-kernel one-shot all-reduce over symmetric peer memory
    (parallel/symm.py) — rank-ordered fp32 sums, so the rollout engine (which fuses the
    decode all-reduce into the row-parallel GEMM and the following residual + RMSNorm) and the
    trainer produce bitwise identical activations;
  * "nccl" (or any torch.distributed backend, e.g. gloo on CPU): dist.all_reduce.

Reference: Megatron tensor / sequence parallel layers used through megatron_utils
(--tensor-model-parallel-size; arguments.py Megatron defaults), SGLang TP engines
(--rollout-num-gpus-per-engine).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from miles_b200.ops._lib import use_native


class TPContext:
    def __init__(self, group, backend: str = "auto", hidden: int = 0, cap_rows: int = 16384):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if backend == "auto":
            backend = "symm" if dist.get_backend(group) == "nccl" else "torch"
        self.backend = backend
        self.hidden = hidden
        self.cap_rows = cap_rows
        self._symm = None

    def symm(self):
        if self._symm is None:
            from miles_b200.parallel.symm import SymmComm

            self._symm = SymmComm(self.group, hidden=self.hidden, cap_rows=self.cap_rows)
        return self._symm

    def use_symm(self, x: torch.Tensor) -> bool:
        return (self.backend == "symm" and x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2
                and x.shape[1] == self.hidden and x.shape[0] <= self.cap_rows)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        if self.use_symm(x):
            return self.symm().all_reduce(x)
        y = x.contiguous().clone()
        dist.all_reduce(y, group=self.group)
        return y

    # ------------------------------------------------------------------ sequence parallel
    def _symm_rows(self, x: torch.Tensor, rows: int) -> bool:
        return (self.backend == "symm" and x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2
                and x.shape[1] == self.hidden and rows <= self.cap_rows)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """Rows of every TP rank, in rank order."""
        if self.size == 1:
            return x
        x = x.contiguous()
        if self._symm_rows(x, x.shape[0]):
            return self.symm().all_gather(x)
        out = x.new_empty((self.size * x.shape[0],) + tuple(x.shape[1:]))
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(out, x, group=self.group)
        else:
            dist.all_gather(list(out.chunk(self.size, 0)), x, group=self.group)
        return out

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's row block of the sum over TP ranks."""
        if self.size == 1:
            return x
        x = x.contiguous()
        R = x.shape[0] // self.size
        if self._symm_rows(x, R):
            return self.symm().reduce_scatter(x)
        if dist.get_backend(self.group) == "nccl":
            out = x.new_empty((R,) + tuple(x.shape[1:]))
            dist.reduce_scatter_tensor(out, x, group=self.group)
            return out
        y = x.clone()
        dist.all_reduce(y, group=self.group)
        return y[self.rank * R:(self.rank + 1) * R].contiguous()

    def local_rows(self, x: torch.Tensor) -> torch.Tensor:
        R = x.shape[0] // self.size
        return x[self.rank * R:(self.rank + 1) * R]

    def shard(self, n: int) -> tuple[int, int]:
        """[lo, hi) of this rank's slice of a dimension of size n."""
        if n % self.size:
            raise ValueError(f"dimension {n} does not split over tensor-parallel size {self.size}")
        s = n // self.size
        return self.rank * s, (self.rank + 1) * s


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return x

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.all_reduce(g.contiguous()), None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        return tp.all_reduce(x)

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    if tp is None or tp.size == 1:
        return x
    return _CopyToTP.apply(x, tp) if torch.is_grad_enabled() and x.requires_grad else x


def reduce_from_tp(x: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    if tp is None or tp.size == 1:
        return x
    if torch.is_grad_enabled() and x.requires_grad:
        return _ReduceFromTP.apply(x, tp)
    return tp.all_reduce(x)


# ------------------------------------------------------------------ parameter layout
_COL = ("self_attn.q_proj.weight", "self_attn.q_b_proj.weight", "self_attn.kv_b_proj.weight",
        "mlp.gate_proj.weight", "mlp.up_proj.weight", "shared_experts.gate_proj.weight",
        "shared_experts.up_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
        "self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias",
        "shared_expert.gate_proj.weight", "shared_expert.up_proj.weight")
_ROW = ("self_attn.o_proj.weight", "mlp.down_proj.weight", "shared_experts.down_proj.weight",
        "shared_expert.down_proj.weight")


def hf_shard_dim(hf_name: str) -> int | None:
    """Dimension along which an HF tensor is split over TP ranks (None: replicated)."""
    if ".experts." in hf_name and "shared_experts" not in hf_name:
        if hf_name.endswith(("gate_proj.weight", "up_proj.weight")):
            return 0
        if hf_name.endswith("down_proj.weight"):
            return 1
        return None
    if hf_name.endswith(_COL):
        return 0
    if hf_name.endswith(_ROW):
        return 1
    return None


def tp_slice(hf_name: str, full: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    if tp is None or tp.size == 1:
        return full
    d = hf_shard_dim(hf_name)
    if d is None:
        return full
    lo, hi = tp.shard(full.shape[d])
    return full.narrow(d, lo, hi - lo)


def _whole_expert(model, name: str) -> bool:
    """Routed-expert tensor (internal or HF name) that is not split over TP (expert_tp = 1)."""
    return (getattr(model, "expert_tp", 0) == 1 and ".experts." in name
            and "shared_experts" not in name)


def model_tp(model, name: str):
    """The TP context that splits parameter `name` of `model` (None: not split)."""
    return None if _whole_expert(model, name) else model.tp


def _gdn_blocks(hf_name: str, cfg):
    """(dim, block sizes) of a Gated DeltaNet tensor in this framework's layout: each block is
    split over TP ranks by heads (key heads, and the value heads each key head serves)."""
    if ".linear_attn." not in hf_name:
        return None
    qk, v = cfg.linear_num_key_heads * cfg.linear_key_head_dim, \
        cfg.linear_num_value_heads * cfg.linear_value_head_dim
    nv = cfg.linear_num_value_heads
    table = {"in_proj_qkvz.weight": (0, [qk, qk, v, v]), "in_proj_qkv.weight": (0, [qk, qk, v]),
             "in_proj_z.weight": (0, [v]), "in_proj_ba.weight": (0, [nv, nv]),
             "in_proj_b.weight": (0, [nv]), "in_proj_a.weight": (0, [nv]),
             "conv1d.weight": (0, [qk, qk, v]), "dt_bias": (0, [nv]), "A_log": (0, [nv]),
             "out_proj.weight": (1, [v])}
    return table.get(hf_name.split(".linear_attn.")[1])


def tp_slice_for(model, hf_name: str, full: torch.Tensor) -> torch.Tensor:
    """This rank's TP slice of a full tensor of `model` (named by its HF name)."""
    tp = model_tp(model, hf_name)
    if tp is None or tp.size == 1:
        return full
    blk = _gdn_blocks(hf_name, model.cfg)
    if blk is None:
        return tp_slice(hf_name, full, tp)
    d, sizes = blk
    parts, off = [], 0
    for n in sizes:
        lo, hi = tp.shard(n)
        parts.append(full.narrow(d, off + lo, hi - lo))
        off += n
    return torch.cat(parts, d)


def tp_gather_for(model, hf_name: str, local: torch.Tensor) -> torch.Tensor:
    """Full tensor of `model` from every TP rank's slice (collective over the TP group)."""
    tp = model_tp(model, hf_name)
    if tp is None or tp.size == 1:
        return local
    blk = _gdn_blocks(hf_name, model.cfg)
    if blk is None:
        return tp_gather(hf_name, local, tp)
    d, sizes = blk
    ranks = [torch.empty_like(local) for _ in range(tp.size)]
    dist.all_gather(ranks, local.contiguous(), group=tp.group)
    split = [n // tp.size for n in sizes]
    per_rank = [r.split(split, d) for r in ranks]
    return torch.cat([per_rank[r][b] for b in range(len(sizes)) for r in range(tp.size)], d)


def tp_partial_param_names(model) -> list[str]:
    """Replicated parameters whose gradient on one TP rank covers only its own slice (its heads,
    its intermediate slice, or under sequence parallelism its rows)."""
    if model.tp is None or model.tp.size == 1:
        return []
    out = []
    # under SP these see only this rank's rows: the norms, and MLA's replicated down projections
    sp_norms = ("input_layernorm.weight", "post_attention_layernorm.weight", "q_a_proj.weight",
                "q_a_layernorm.weight", "kv_a_proj_with_mqa.weight", "kv_a_layernorm.weight",
                "post_self_attn_layernorm.weight", "post_mlp_layernorm.weight")
    for name in model.params:
        if name.endswith(("self_attn.q_norm.weight", "self_attn.k_norm.weight", "linear_attn.norm.weight")):
            out.append(name)
        elif (model.sequence_parallel and model.cp is None
              and (name.endswith(sp_norms) or name == "norm.weight")):
            out.append(name)
        elif model.vocab_parallel_logprob and model.cp is None and name == "lm_head.weight":
            out.append(name)  # each rank's gradient covers its vocabulary rows
        elif name.endswith(("mlp.gate.weight", "mlp.shared_expert_gate.weight")):
            out.append(name)  # gate logits scale partial expert outputs
        elif model.ep is None and _whole_expert(model, name):
            out.append(name)  # whole experts on every TP rank, each fed its own rows
    return out


def tp_gather(hf_name: str, local: torch.Tensor, tp: TPContext | None) -> torch.Tensor:
    """Full tensor from every rank's slice (collective over the TP group)."""
    if tp is None or tp.size == 1:
        return local
    d = hf_shard_dim(hf_name)
    if d is None:
        return local
    parts = [torch.empty_like(local) for _ in range(tp.size)]
    dist.all_gather(parts, local.contiguous(), group=tp.group)
    return torch.cat(parts, d)


_SHARDED_INTERNAL = ("self_attn.qkv_proj.weight", "self_attn.o_proj.weight", "mlp.gate_up_proj.weight",
                     "mlp.down_proj.weight", "mlp.experts.w1", "mlp.experts.w2",
                     "shared_experts.gate_up_proj.weight", "shared_experts.down_proj.weight",
                     "self_attn.q_proj.weight", "self_attn.q_b_proj.weight",
                     "self_attn.kv_b_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                     "self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias",
                     "shared_expert.gate_up_proj.weight", "shared_expert.down_proj.weight",
                     "linear_attn.in_proj_qkvz.weight", "linear_attn.in_proj_ba.weight",
                     "linear_attn.conv1d.weight", "linear_attn.dt_bias", "linear_attn.A_log",
                     "linear_attn.out_proj.weight")


def is_tp_sharded(name: str) -> bool:
    """True for internal parameter names that tensor parallelism splits."""
    return name.endswith(_SHARDED_INTERNAL)


def tp_replicated_ranges(model) -> list[tuple[int, int]]:
    """Flat-buffer ranges of the parameters every TP rank holds in full."""
    if model.tp is None or model.tp.size == 1:
        return []
    return [(s.offset, s.offset + s.numel) for s in model.specs
            if not s.name.endswith(_SHARDED_INTERNAL) or (model.ep is None and _whole_expert(model, s.name))]



# ------------------------------------------------------------------ sequence parallel
# Under sequence parallelism the residual stream, norms and embeddings hold T / tp rows per
# rank; column-parallel projections take the all-gathered rows, row-parallel projections end
# in a reduce-scatter (fused into the GEMM epilogue with the symmetric-memory backend).
class _SPGather(torch.autograd.Function):
    """Forward all-gather rows; backward reduce-scatter."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.all_gather(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.reduce_scatter(g), None


class _SPReduceScatter(torch.autograd.Function):
    """Forward reduce-scatter rows; backward all-gather."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.reduce_scatter(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.all_gather(g), None


class _SPSplit(torch.autograd.Function):
    """Forward: this rank's rows of a replicated tensor; backward all-gather (so the gradient of
    the replicated input is complete and identical on every rank)."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.local_rows(x).contiguous()

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.all_gather(g.contiguous()), None


class _SPGatherReplicated(torch.autograd.Function):
    """Forward all-gather rows into a tensor every rank then uses identically; backward keeps
    this rank's rows of the (identical) gradient."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.all_gather(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.local_rows(g).contiguous(), None


class _RowParallelRS(torch.autograd.Function):
    """y_local = reduce_scatter(x @ w^T) with the GEMM's epilogue storing each output row into
    its owner's staging (symmetric-memory backend); backward all-gathers dy."""

    @staticmethod
    def forward(ctx, x, w, tp):
        ctx.tp = tp
        ctx.save_for_backward(x, w)
        return tp.symm().gemm_reduce_scatter(x, w)

    @staticmethod
    def backward(ctx, g):
        from miles_b200.ops import gemm as G

        x, w = ctx.saved_tensors
        dy = ctx.tp.all_gather(g.contiguous())
        dx = G.matmul_nn(dy, w)
        dw = G._accumulate_wgrad(w, dy, x) if ctx.needs_input_grad[1] else None
        return dx, dw, None


def sp_gather(x, tp):
    if tp is None or tp.size == 1:
        return x
    return _SPGather.apply(x, tp) if torch.is_grad_enabled() and x.requires_grad else tp.all_gather(x)


def sp_reduce_scatter(x, tp):
    if tp is None or tp.size == 1:
        return x
    if torch.is_grad_enabled() and x.requires_grad:
        return _SPReduceScatter.apply(x, tp)
    return tp.reduce_scatter(x)


def sp_split(x, tp):
    if tp is None or tp.size == 1:
        return x
    if torch.is_grad_enabled() and x.requires_grad:
        return _SPSplit.apply(x, tp)
    return tp.local_rows(x).contiguous()


def sp_gather_replicated(x, tp):
    if tp is None or tp.size == 1:
        return x
    if torch.is_grad_enabled() and x.requires_grad:
        return _SPGatherReplicated.apply(x, tp)
    return tp.all_gather(x)


def row_parallel_rs(x, w, tp, lin):
    """reduce_scatter(x @ w^T): fused GEMM + reduce-scatter when the symmetric-memory backend
    covers the shape, else `lin(x, w)` followed by the reduce-scatter collective."""
    if tp is not None and tp.size > 1 and tp.backend == "symm" and x.is_cuda \
            and x.shape[0] // tp.size <= tp.cap_rows and w.shape[0] == tp.hidden:
        return _RowParallelRS.apply(x, w, tp)
    return sp_reduce_scatter(lin(x, w), tp)


# ------------------------------------------------------------------ vocab-parallel log-prob
class _VocabParallelLogProb(torch.autograd.Function):
    """log softmax(h W^T / T)[target] and the entropy with every TP rank computing the logits of
    its vocabulary slice only: the row max, the sum of exponentials, the target logit and
    sum(p z) are combined over the TP group (max / sum all-reduces), so no rank holds [n, V]
    logits. Backward: each rank forms the logit gradient of its slice; the hidden-state gradient
    is a partial sum (the caller's copy_to_tp all-reduces it) and the LM-head gradient lands in
    this rank's rows (tp_partial_param_names all-reduces it)."""

    @staticmethod
    def forward(ctx, h, W, targets, inv_temp, tp, lo, hi, chunk):
        from miles_b200.ops import gemm as G

        n = h.shape[0]
        lp = torch.empty(n, dtype=torch.float32, device=h.device)
        ent = torch.empty_like(lp)
        lse = torch.empty_like(lp)
        Wl = W[lo:hi]
        ctx.save_for_backward(h, W, targets, lse, ent)
        ctx.cfg = (inv_temp, lo, hi, chunk)
        if use_native(h):
            _vp_logprob_fwd(h, Wl, targets, inv_temp, tp, lo, chunk, lp, ent, lse)
            return lp, ent
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            z = G.matmul_nt(h[s:e].contiguous(), Wl, out_dtype=torch.float32) * inv_temp
            m = z.max(-1).values
            dist.all_reduce(m, op=dist.ReduceOp.MAX, group=tp.group)
            ex = torch.exp(z - m[:, None])
            se = ex.sum(-1)
            tgt = targets[s:e].long()
            inr = (tgt >= lo) & (tgt < hi)
            tz = torch.where(inr, z.gather(1, (tgt - lo).clamp(0, hi - lo - 1)[:, None])[:, 0],
                             torch.zeros_like(m))
            pz = (ex * z).sum(-1)
            red = torch.stack([se, tz, pz], 0)
            dist.all_reduce(red, group=tp.group)
            l = m + torch.log(red[0])
            lse[s:e] = l
            lp[s:e] = red[1] - l
            ent[s:e] = l - red[2] / red[0]
        return lp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):
        from miles_b200.ops import gemm as G

        h, W, targets, lse, ent = ctx.saved_tensors
        inv_temp, lo, hi, chunk = ctx.cfg
        n = h.shape[0]
        Wl = W[lo:hi]
        if use_native(h):
            dh, dW = _vp_logprob_bwd(h, W, targets, inv_temp, lo, hi, chunk, lse, ent, g_lp, g_ent,
                                     ctx.needs_input_grad[1])
            return dh, dW, None, None, None, None, None, None
        dh = torch.empty(h.shape, dtype=torch.float32, device=h.device)
        dW = torch.zeros(W.shape, dtype=torch.float32, device=h.device) if ctx.needs_input_grad[1] else None
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            hs = h[s:e].contiguous()
            z = G.matmul_nt(hs, Wl, out_dtype=torch.float32) * inv_temp
            p = torch.exp(z - lse[s:e, None])
            dz = torch.zeros_like(z)
            if g_lp is not None:
                tgt = targets[s:e].long()
                inr = (tgt >= lo) & (tgt < hi)
                onehot = torch.zeros_like(z)
                idx = (tgt - lo).clamp(0, hi - lo - 1)
                onehot.scatter_(1, idx[:, None], inr[:, None].float())
                dz += g_lp[s:e, None] * (onehot - p)
            if g_ent is not None:
                dz += g_ent[s:e, None] * (-p * (z - lse[s:e, None] + ent[s:e, None]))
            dz = dz * inv_temp
            dh[s:e] = dz @ Wl.float()
            if dW is not None:
                dW[lo:hi] += dz.t() @ hs.float()
        return dh.to(h.dtype), (dW.to(W.dtype) if dW is not None else None), None, None, None, None, None, None


def _vp_logprob_fwd(h, Wl, targets, inv_temp, tp, lo, chunk, lp, ent, lse):
    """Kernel path of the vocabulary-parallel forward, per row chunk: the tcgen05 GEMM writes this
    rank's fp32 logit slice, one kernel reduces it to the slice's softmax statistics
    {max, sum exp, sum exp * z, target logit} (csrc/rl_ops.cu logprob_part_kernel), ONE
    all-gather exchanges those 4 floats per row, and a second kernel combines the ranks' parts in
    rank order into lse / log-prob / entropy (logprob_combine_kernel: every rank gets the same
    bits; with one rank it is exactly the single-GPU log-prob kernel)."""
    from miles_b200.ops import gemm as G
    from miles_b200.ops._lib import lib

    n = h.shape[0]
    V = Wl.shape[0]
    world = tp.size
    cs = min(chunk, max(n, 1))
    zbuf = torch.empty(cs, V, dtype=torch.float32, device=h.device)
    part = torch.empty(4, cs, dtype=torch.float32, device=h.device)
    parts = torch.empty(world, 4, cs, dtype=torch.float32, device=h.device)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        k = e - s
        z = zbuf[:k]
        G.matmul_nt(h[s:e].contiguous(), Wl, out=z)
        pk = part[:, :k] if k == cs else torch.empty(4, k, dtype=torch.float32, device=h.device)
        lib().logprob_part(z, targets[s:e], lo, inv_temp, pk)
        pa = parts if k == cs else torch.empty(world, 4, k, dtype=torch.float32, device=h.device)
        dist.all_gather_into_tensor(pa, pk, group=tp.group)
        lib().logprob_combine(pa, world, lp[s:e], ent[s:e], lse[s:e])


def _vp_logprob_bwd(h, W, targets, inv_temp, lo, hi, chunk, lse, ent, g_lp, g_ent, need_dw):
    """Kernel path of the vocabulary-parallel backward: the logit gradient of this rank's slice
    (csrc/rl_ops.cu logprob_bwd_kernel with the global lse / entropy and slice-relative targets,
    bf16), then the GEMMs for the partial hidden-state gradient and this slice's LM-head rows."""
    from miles_b200.ops import gemm as G
    from miles_b200.ops._lib import lib

    n, H = h.shape
    Wl = W[lo:hi]
    V = hi - lo
    cs = min(chunk, max(n, 1))
    dh = torch.empty_like(h)
    dW = torch.zeros(W.shape, dtype=torch.float32, device=h.device) if need_dw else None
    zbuf = torch.empty(cs, V, dtype=torch.float32, device=h.device)
    dbuf = torch.empty(cs, V, dtype=torch.bfloat16, device=h.device)
    tl = (targets - lo).int().contiguous()  # outside the slice: never equal to a slice index
    g_lp = g_lp.contiguous() if g_lp is not None else None
    g_ent = g_ent.contiguous() if g_ent is not None else None
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        hs = h[s:e].contiguous()
        z, d = zbuf[:e - s], dbuf[:e - s]
        G.matmul_nt(hs, Wl, out=z)
        lib().logprob_bwd(z, tl[s:e], inv_temp, lse[s:e], None if g_lp is None else g_lp[s:e],
                          None if g_ent is None else g_ent[s:e], ent[s:e], d)
        G.matmul_nn(d, Wl, out=dh[s:e])
        if dW is not None:
            G.matmul_tn(d, hs, out=dW[lo:hi], accumulate=True)
    return dh, (dW.to(W.dtype) if dW is not None else None)


def vocab_parallel_logprob(h, W, targets, temperature: float, tp: TPContext, chunk: int = 4096):
    """(log-prob, entropy) of `targets` with the vocabulary split over the TP group; `h` must be
    identical on every TP rank (it is passed through copy_to_tp here)."""
    lo, hi = tp.shard(W.shape[0])
    return _VocabParallelLogProb.apply(copy_to_tp(h, tp), W, targets.int().contiguous(),
                                       1.0 / temperature, tp, lo, hi, chunk)
