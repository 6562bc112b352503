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

Interleaved schedule (`vpp` > 1, `run_interleaved`): each rank holds vpp model chunks, a
micro-batch passes every rank vpp times, and the bubble shrinks to (P - 1) / vpp stage-times.

Reference: Megatron get_forward_backward_func 1F1B (megatron_utils/model.py:440-450), virtual
pipeline size (megatron_utils/initialize.py:44),
--pipeline-model-parallel-size, loss on the last stage (model.py:487-490), PP shards gathered
at refit (update_weight/common.py).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


_TIED_GROUPS: dict = {}


def stage_layer_counts(num_layers: int, n_stages: int, first: int | None = None,
                       last: int | None = None) -> list[int]:
    """Layers per (virtual) stage: `first` / `last` pin the first and last stage's counts (the
    embedding / LM-head stages often take fewer layers), the rest are split evenly with the
    remainder on the earlier stages."""
    head = [first] if first is not None else []
    tail = [last] if last is not None else []
    mid_n = n_stages - len(head) - len(tail)
    rest = num_layers - sum(head) - sum(tail)
    if mid_n < 0 or rest < 0 or (mid_n == 0 and rest != 0):
        raise ValueError(f"first={first} / last={last} layers do not fit {num_layers} layers "
                         f"in {n_stages} stages")
    base, extra = divmod(rest, mid_n) if mid_n else (0, 0)
    return head + [base + (1 if v < extra else 0) for v in range(mid_n)] + tail


class PPContext:
    """Stage layout of one pipeline. With `vpp` > 1 (interleaved / virtual pipeline) the layers
    are cut into size * vpp chunks; rank s owns chunks c * size + s for c < vpp, so a
    micro-batch visits every rank vpp times (model chunk c of rank s is virtual stage
    c * size + s)."""

    def __init__(self, group, num_layers: int, vpp: int = 1, first_layers: int | None = None,
                 last_layers: int | None = None):
        self.group = group
        self.size = dist.get_world_size(group)
        self.stage = dist.get_rank(group)
        self.vpp = vpp
        nv = self.size * vpp
        counts = stage_layer_counts(num_layers, nv, first_layers, last_layers)
        if min(counts) == 0:
            raise ValueError(f"{num_layers} layers do not fill {nv} (virtual) pipeline stages")
        self.vbounds = [sum(counts[:v]) for v in range(nv + 1)]
        # layer ranges of this rank's model chunks, in chunk order
        self.chunks = [(self.vbounds[c * self.size + self.stage], self.vbounds[c * self.size + self.stage + 1])
                       for c in range(vpp)]
        self.layer_ids = [i for lo, hi in self.chunks for i in range(lo, hi)]
        if vpp == 1:
            self.bounds = self.vbounds
            self.lo, self.hi = self.chunks[0]
        self.is_first = self.stage == 0
        self.is_last = self.stage == self.size - 1
        self.ranks = [dist.get_global_rank(group, s) for s in range(self.size)]
        key = tuple(self.ranks)
        if key not in _TIED_GROUPS and self.size > 1 and self.size == dist.get_world_size():
            # one pipeline spans the job: create its first/last-stage group here (new_group is
            # collective over the job; with several pipelines the launcher creates them all)
            from miles_b200.parallel.reloadable import REGISTRY

            _TIED_GROUPS[key] = REGISTRY.new_group([self.ranks[0], self.ranks[-1]])

    def stage_of_layer(self, i: int) -> int:
        """Rank (within the pipeline group) that owns layer i."""
        for v in range(self.size * self.vpp):
            if self.vbounds[v] <= i < self.vbounds[v + 1]:
                return v % self.size
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


def _virtual_order(P: int, V: int, n_mb: int, reverse: bool) -> list[tuple[int, int]]:
    """(micro-batch, chunk) visit order of one rank: groups of P micro-batches go through chunk
    0, 1, ..., V-1 (backwards: V-1, ..., 0) before the next group starts."""
    out = []
    for g in range(0, n_mb, P):
        grp = range(g, min(g + P, n_mb))
        for c in (reversed(range(V)) if reverse else range(V)):
            out += [(j, c) for j in grp]
    return out


def interleaved_schedule(P: int, V: int, n_mb: int, train: bool = True):
    """Plan of the interleaved 1F1B schedule for every rank of a P-stage pipeline with V model
    chunks per rank, as a list of ticks.

    Each rank runs its own op sequence: forwards in `_virtual_order`, of which the first
    (P - s - 1) * 2 + (V - 1) * P are warm-up, then alternating one forward / one backward,
    then the remaining backwards. The plan is found by simulating all ranks in lockstep: in a
    tick each rank runs its next op if its input was produced in an earlier tick. An op's
    message (activation to virtual stage v+1, gradient to v-1) is exchanged at the end of the
    tick that produced it, so every rank derives the same (sender, receiver) pairs per tick
    and posts them in one batched send/recv: no ordering of point-to-point calls can
    deadlock. If the warm-up depth of the 1F1B order stalls (possible when n_mb is not a
    multiple of P), every rank falls back to all forwards, then all backwards.

    Returns ticks: list of (ops, msgs) with ops {rank: ("F" | "B", mb, chunk)} and msgs
    [(src, dst, "F" | "B", mb, v_dst)], v_dst the virtual stage that consumes the message."""
    NV = P * V

    def seqs(warm_fn):
        out = []
        for s in range(P):
            fw = _virtual_order(P, V, n_mb, False)
            if not train:
                out.append([("F", j, c) for j, c in fw])
                continue
            bw = _virtual_order(P, V, n_mb, True)
            w = min(warm_fn(s), len(fw))
            ops = [("F", j, c) for j, c in fw[:w]]
            fi, bi = w, 0
            while fi < len(fw):
                ops.append(("F",) + fw[fi]); fi += 1
                ops.append(("B",) + bw[bi]); bi += 1
            ops += [("B",) + x for x in bw[bi:]]
            out.append(ops)
        return out

    def simulate(per_rank):
        done: dict = {}
        pos = [0] * P
        ticks = []
        t = 0
        while any(pos[s] < len(per_rank[s]) for s in range(P)):
            ops, msgs = {}, []
            for s in range(P):
                if pos[s] >= len(per_rank[s]):
                    continue
                kind, j, c = per_rank[s][pos[s]]
                v = c * P + s
                if kind == "F":
                    dep = [("F", j, v - 1)] if v > 0 else []
                else:
                    dep = [("F", j, v)] + ([("B", j, v + 1)] if v < NV - 1 else [])
                if all(done.get(d, t) < t for d in dep):
                    ops[s] = (kind, j, c)
            if not ops:
                return None
            for s, (kind, j, c) in ops.items():
                v = c * P + s
                done[(kind, j, v)] = t
                pos[s] += 1
                if kind == "F" and v < NV - 1:
                    msgs.append((s, (v + 1) % P, "F", j, v + 1))
                if kind == "B" and v > 0:
                    msgs.append((s, (v - 1) % P, "B", j, v - 1))
            ticks.append((ops, msgs))
            t += 1
        return ticks

    warm = (lambda s: (P - s - 1) * 2 + (V - 1) * P) if V > 1 else (lambda s: P - s - 1)
    plan = simulate(seqs(warm))
    if plan is None:
        plan = simulate(seqs(lambda s: n_mb * V))
    return plan


def run_interleaved(pp: PPContext, n_mb: int, shapes: list[tuple], dtype, device,
                    forward: Callable[[int, int, torch.Tensor | None], torch.Tensor],
                    backward: Callable[[int, int, torch.Tensor, torch.Tensor | None], None] | None) -> None:
    """Drive `n_mb` micro-batches through this rank's `pp.vpp` model chunks.

    forward(j, c, h_in) -> output of chunk c for micro-batch j (the loss on the last virtual
    stage); h_in None on virtual stage 0. backward(j, c, output, grad) (grad None on the last
    virtual stage); backward None runs the forward-only schedule (log-probs)."""
    P, V, me = pp.size, pp.vpp, pp.stage
    plan = interleaved_schedule(P, V, n_mb, train=backward is not None)
    mail: dict = {}
    saved: dict = {}
    pending: dict = {}
    for ops, msgs in plan:
        op = ops.get(me)
        if op is not None:
            kind, j, c = op
            v = c * P + me
            if kind == "F":
                h = mail.pop(("F", j, v), None)
                if h is not None and backward is not None:
                    h.requires_grad_(True)
                out = forward(j, c, h)
                if backward is not None:
                    saved[(j, c)] = (h, out)
                pending[("F", j, v + 1)] = out
            else:
                h, out = saved.pop((j, c))
                backward(j, c, out, mail.pop(("B", j, v), None))
                pending[("B", j, v - 1)] = h.grad if h is not None else None
        p2p = []
        for src, dst, kind, j, vd in msgs:
            if src == me:
                t = pending.pop((kind, j, vd))
                t = (t.detach() if kind == "F" else t).contiguous()
                p2p.append(dist.P2POp(dist.isend, t, pp.ranks[dst], group=pp.group))
            elif dst == me:
                t = torch.empty(shapes[j], dtype=dtype, device=device)
                mail[(kind, j, vd)] = t
                p2p.append(dist.P2POp(dist.irecv, t, pp.ranks[src], group=pp.group))
        _p2p(p2p)
        pending = {k: t for k, t in pending.items() if t is not None and k[2] not in (-1, P * V)}


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
        from miles_b200.parallel.reloadable import REGISTRY

        _TIED_GROUPS[tuple(ranks)] = REGISTRY.new_group([ranks[0], ranks[-1]])


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
