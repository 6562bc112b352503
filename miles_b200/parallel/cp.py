"""Context parallelism for the training forward (long sequences).

Each rank of a CP group of size c holds T / c consecutive rows of the packed micro-batch (the
batch is padded to a multiple of c). Everything but attention is per token and runs on the
local rows. Attention needs every key of a sequence, so around it the rows are exchanged by
head: an all-to-all turns [T/c rows, all heads] into [all T rows, heads / c] (every rank then
runs the ordinary varlen attention kernel for its head slice over the whole batch), and a
second all-to-all turns the output back. The per-head arithmetic is unchanged, so the result
is bitwise the forward without CP (and the rollout engine's log-probs stay exact).

The exchange moves 4 x T x heads x D elements per layer in the forward (q, k, v, o), which on
NVLink is small next to the attention itself. With fewer KV heads than ranks (c a multiple of
the KV-head count, GQA), each KV head is replicated c / nkv times before the exchange, so every
rank receives the one KV head that its query heads attend to; the forward arithmetic is still
that of the run without CP, and the backward of the replication sums the replicas' gradients.
So CP is not capped at the KV-head count (4 KV heads of Qwen3-30B-A3B, CP 8).

Gradients: each rank's parameter gradients cover its own rows, so the optimizer reduces them
over data-parallel x context-parallel ranks. The per-token log-probs are computed on the rows
each rank holds and all-gathered (backward: each rank keeps its own part), so the loss is
evaluated identically on every CP rank while each LM-head gradient term is counted once.

Reference: Megatron context parallelism (--context-parallel-size; cp_utils.py zigzag split,
ring attention through TE) and the allgather-CP variant (--allgather-cp). The head
all-to-all is a different exchange with the same result.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class CPContext:
    def __init__(self, group):
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def rows(self, T: int) -> tuple[int, int, int]:
        """(padded total, lo, hi) of this rank's rows."""
        Tp = (T + self.size - 1) // self.size * self.size
        R = Tp // self.size
        return Tp, self.rank * R, (self.rank + 1) * R


def _a2a(x: torch.Tensor, group) -> torch.Tensor:
    out = torch.empty_like(x)
    dist.all_to_all_single(out, x.contiguous(), group=group)
    return out


class _TokensToHeads(torch.autograd.Function):
    """[R, nh, D] local rows, all heads -> [c*R, nh/c, D] all rows, this rank's heads."""

    @staticmethod
    def forward(ctx, x, cp):
        ctx.cp = cp
        return _tokens_to_heads(x, cp)

    @staticmethod
    def backward(ctx, g):
        return _heads_to_tokens(g, ctx.cp), None


class _HeadsToTokens(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, cp):
        ctx.cp = cp
        return _heads_to_tokens(x, cp)

    @staticmethod
    def backward(ctx, g):
        return _tokens_to_heads(g, ctx.cp), None


def _tokens_to_heads(x, cp):
    R, nh, D = x.shape
    c = cp.size
    send = x.reshape(R, c, nh // c, D).transpose(0, 1).contiguous()  # [c (dest), R, nh/c, D]
    recv = _a2a(send, cp.group)                                       # [c (source), R, nh/c, D]
    return recv.reshape(c * R, nh // c, D)


def _heads_to_tokens(x, cp):
    T, hl, D = x.shape
    c = cp.size
    R = T // c
    send = x.reshape(c, R, hl, D).contiguous()                        # [c (dest rows), R, hl, D]
    recv = _a2a(send, cp.group)                                       # [c (source heads), R, hl, D]
    return recv.transpose(0, 1).reshape(R, c * hl, D)


def kv_tokens_to_heads(x, cp):
    """tokens_to_heads for K / V: with fewer KV heads than ranks (cp.size a multiple of them),
    replicate each KV head cp.size / nkv times first, so rank r gets KV head r // (cp.size / nkv),
    the one its query heads [r * nq / c, (r + 1) * nq / c) use."""
    nh = x.shape[1]
    c = cp.size
    if nh % c == 0:
        return tokens_to_heads(x, cp)
    if c % nh:
        raise ValueError(f"{nh} KV heads neither split over nor divide CP {c}")
    return tokens_to_heads(x.repeat_interleave(c // nh, dim=1), cp)


def tokens_to_heads(x, cp):
    if torch.is_grad_enabled() and x.requires_grad:
        return _TokensToHeads.apply(x, cp)
    return _tokens_to_heads(x, cp)


@torch.no_grad()
def all_gather_rows(x: torch.Tensor, cp) -> torch.Tensor:
    """Every CP rank's rows of x, concatenated in rank order (no gradient)."""
    parts = [torch.empty_like(x) for _ in range(cp.size)]
    dist.all_gather(parts, x.contiguous(), group=cp.group)
    return torch.cat(parts, 0)


def heads_to_tokens(x, cp):
    if torch.is_grad_enabled() and x.requires_grad:
        return _HeadsToTokens.apply(x, cp)
    return _heads_to_tokens(x, cp)


class _GatherParts(torch.autograd.Function):
    """Concatenate every rank's 1-D part (sizes known on every rank); backward keeps this rank's
    slice of the (identical) gradient."""

    @staticmethod
    def forward(ctx, x, cp, sizes):
        ctx.cp, ctx.sizes = cp, sizes
        m = max(sizes)
        buf = torch.zeros(m, dtype=x.dtype, device=x.device)
        buf[: x.numel()] = x
        parts = [torch.empty(m, dtype=x.dtype, device=x.device) for _ in range(cp.size)]
        dist.all_gather(parts, buf, group=cp.group)
        return torch.cat([p[:n] for p, n in zip(parts, sizes)])

    @staticmethod
    def backward(ctx, g):
        lo = sum(ctx.sizes[: ctx.cp.rank])
        return g[lo:lo + ctx.sizes[ctx.cp.rank]].contiguous(), None, None


def gather_parts(x: torch.Tensor, cp: CPContext, sizes: list[int]) -> torch.Tensor:
    return _GatherParts.apply(x, cp, sizes)
