"""Pipeline parallelism for training: layer stages, the 1F1B schedule over NCCL point-to-point,
and the weight gather that feeds a full-model rollout engine.

Stage s of a pipeline of P stages owns layers [s*L/P, (s+1)*L/P) (the remainder goes to the
first stages), the embedding on stage 0 and the final norm + LM head on stage P-1 (with tied
embeddings the last stage keeps a copy of the embedding whose gradient is summed with stage 0's).
Between stages flows the residual stream [T, H] of every micro-batch, and its gradient back.

Schedule (non-interleaved 1F1B): stage s runs P-s-1 warm-up forwards, then alternates one
forward and one backward, then drains the remaining backwards. Each steady-state step pairs its
send and receive in one batched isend/irecv (send the forward output while receiving the
gradient of an earlier micro-batch, and the reverse), so no ordering of blocking sends can
deadlock. The loss lives on the last stage.

Reference: Megatron get_forward_backward_func 1F1B (megatron_utils/model.py:440-450),
--pipeline-model-parallel-size, loss on the last stage (model.py:487-490), PP shards gathered
at refit (update_weight/common.py).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


_TIED_GROUPS: dict = {}


class PPContext:
    def __init__(self, group, num_layers: int):
        self.group = group
        self.size = dist.get_world_size(group)
        self.stage = dist.get_rank(group)
        base, extra = divmod(num_layers, self.size)
        counts = [base + (1 if s < extra else 0) for s in range(self.size)]
        if min(counts) == 0:
            raise ValueError(f"{num_layers} layers do not fill {self.size} pipeline stages")
        self.bounds = [sum(counts[:s]) for s in range(self.size + 1)]
        self.lo, self.hi = self.bounds[self.stage], self.bounds[self.stage + 1]
        self.is_first = self.stage == 0
        self.is_last = self.stage == self.size - 1
        self.ranks = [dist.get_global_rank(group, s) for s in range(self.size)]
        key = tuple(self.ranks)
        if key not in _TIED_GROUPS and self.size > 1 and self.size == dist.get_world_size():
            # one pipeline spans the job: create its first/last-stage group here (new_group is
            # collective over the job; with several pipelines the launcher creates them all)
            _TIED_GROUPS[key] = dist.new_group([self.ranks[0], self.ranks[-1]])

    def stage_of_layer(self, i: int) -> int:
        for s in range(self.size):
            if self.bounds[s] <= i < self.bounds[s + 1]:
                return s
        raise IndexError(i)

    @property
    def prev(self) -> int:
        return self.ranks[self.stage - 1]

    @property
    def next(self) -> int:
        return self.ranks[self.stage + 1]


def _p2p(ops):
    if ops:
        for r in dist.batch_isend_irecv(ops):
            r.wait()


def run_1f1b(pp: PPContext, n_mb: int, shapes: list[tuple], dtype, device,
             forward: Callable[[int, torch.Tensor | None], torch.Tensor],
             backward: Callable[[int, torch.Tensor, torch.Tensor | None], None]) -> None:
    """Drive `n_mb` micro-batches through this stage.

    forward(j, h_in) -> output (the residual stream to send on, or the loss on the last stage);
    h_in is None on the first stage, else the received hidden (requires grad).
    backward(j, output, grad) runs the backward of micro-batch j (grad None on the last stage).
    shapes[j]: shape of the hidden exchanged for micro-batch j."""
    first, last = pp.is_first, pp.is_last
    warm = min(pp.size - pp.stage - 1, n_mb)
    rem = n_mb - warm
    saved: dict[int, tuple] = {}

    def recv(j, src):
        t = torch.empty(shapes[j], dtype=dtype, device=device)
        return t, dist.P2POp(dist.irecv, t, src, group=pp.group)

    def run_fwd(j, h):
        if h is not None:
            h.requires_grad_(True)
        out = forward(j, h)
        saved[j] = (h, out)
        return out

    def run_bwd(j, g):
        h, out = saved.pop(j)
        backward(j, out, g)
        return h.grad if h is not None else None

    # warm-up forwards
    for j in range(warm):
        h = None
        if not first:
            h, op = recv(j, pp.prev)
            _p2p([op])
        out = run_fwd(j, h)
        if not last:
            _p2p([dist.P2POp(dist.isend, out.detach().contiguous(), pp.next, group=pp.group)])
    # steady state
    h = None
    if rem > 0 and not first:
        h, op = recv(warm, pp.prev)
        _p2p([op])
    for i in range(rem):
        j = warm + i
        out = run_fwd(j, h)
        g = None
        if not last:
            g, op = recv(i, pp.next)
            _p2p([dist.P2POp(dist.isend, out.detach().contiguous(), pp.next, group=pp.group), op])
        dh = run_bwd(i, g)
        h = None
        if i == rem - 1:
            if not first:
                _p2p([dist.P2POp(dist.isend, dh.contiguous(), pp.prev, group=pp.group)])
        else:
            ops = []
            if not first:
                h, op = recv(j + 1, pp.prev)
                ops = [dist.P2POp(dist.isend, dh.contiguous(), pp.prev, group=pp.group), op]
            _p2p(ops)
    # cool-down backwards
    for i in range(rem, n_mb):
        g = None
        if not last:
            g, op = recv(i, pp.next)
            _p2p([op])
        dh = run_bwd(i, g)
        if not first:
            _p2p([dist.P2POp(dist.isend, dh.contiguous(), pp.prev, group=pp.group)])


def run_forward_only(pp: PPContext, n_mb: int, shapes: list[tuple], dtype, device,
                     forward: Callable[[int, torch.Tensor | None], torch.Tensor]) -> None:
    """Forward-only pipeline (log-probs of old / reference policies)."""
    for j in range(n_mb):
        h = None
        if not pp.is_first:
            h = torch.empty(shapes[j], dtype=dtype, device=device)
            dist.recv(h, pp.prev, group=pp.group)
        out = forward(j, h)
        if not pp.is_last:
            dist.send(out.contiguous(), pp.next, group=pp.group)


def reduce_tied_embedding(model) -> None:
    """With tied embeddings the first and last stages both hold the embedding: sum their
    gradients (the update is then identical on both)."""
    pp = model.pp
    if pp is None or not model.cfg.tie_embeddings or pp.size == 1:
        return
    if pp.is_first or pp.is_last:
        g = model.params["embed_tokens.weight"].main_grad
        grp = tied_embedding_group(pp)
        dist.all_reduce(g, group=grp)


@torch.no_grad()
def sync_tied_embedding(model) -> None:
    """Make the last stage's embedding copy equal to stage 0's."""
    pp = model.pp
    if pp is None or pp.size == 1 or not model.cfg.tie_embeddings:
        return
    if pp.is_first or pp.is_last:
        dist.broadcast(model.params["embed_tokens.weight"].data, pp.ranks[0],
                       group=tied_embedding_group(pp))


def tied_embedding_group(pp: PPContext):
    """Group of the first and last stage ranks of this pipeline."""
    return _TIED_GROUPS[tuple(pp.ranks)]


def register_tied_embedding_groups(world: int, pp_size: int) -> None:
    """Create the first/last-stage group of every pipeline (pipelines are strided rank sets
    {d, d + D, ...} with D = world / pp_size); collective, call on every rank."""
    D = world // pp_size
    for d in range(D):
        ranks = [d + s * D for s in range(pp_size)]
        _TIED_GROUPS[tuple(ranks)] = dist.new_group([ranks[0], ranks[-1]])


@torch.no_grad()
def gather_full_weights(stage_model, full_model) -> None:
    """Copy every stage's parameters into `full_model` (a full-depth Transformer on every rank
    of the pipeline group, e.g. the rollout engine's): each parameter is broadcast from the
    stage that owns it."""
    pp = stage_model.pp
    for name, p in full_model.params.items():
        if name.startswith("layers."):
            owner = pp.stage_of_layer(int(name.split(".")[1]))
        elif name == "embed_tokens.weight":
            owner = 0
        else:
            owner = pp.size - 1
        src = stage_model.params[name].data if pp.stage == owner else p.data
        buf = src.contiguous() if pp.stage == owner else torch.empty_like(p.data)
        dist.broadcast(buf, pp.ranks[owner], group=pp.group)
        p.data.copy_(buf)
    full_model.weight_version = stage_model.weight_version
