"""Prefill / decode disaggregation between rollout engines on different ranks.

A prefill rank runs `RolloutEngine.prefill_handoffs(requests)` (packed prefill and the first
sampled token) and sends the hand-offs to a decode rank, which continues them with
`RolloutEngine.generate(handoffs)`: the prompt's K/V rows are copied into its own pages, so it
never recomputes the prompt. Both engines run the same batch-invariant kernels, so the decode
rank produces the tokens, log-probs and routing a single engine would.

Transport: one object message (requests, first tokens, shapes, routing) and one flat tensor
with every K/V row, over torch.distributed point-to-point (NCCL over NVLink between GPUs,
gloo on CPU ranks).

Reference roles: the SGLang prefill / decode server groups of the deployment config
(miles/backends/sglang_utils/sglang_config.py:169-186, `worker_type: prefill | decode`) and
their KV transfer.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from miles_b200.engine.engine import PrefillHandoff


def send_handoffs(handoffs: list[PrefillHandoff], dst: int, group=None) -> int:
    """Send hand-offs to global rank `dst`; returns the K/V bytes sent."""
    meta = [(h.req, h.token, h.logprob, [tuple(t.shape) for t in h.k], str(h.k[0].dtype) if h.k else "",
             h.experts) for h in handoffs]
    dev = handoffs[0].k[0].device if handoffs and handoffs[0].k else None
    dist.send_object_list([meta], dst=dst, group=group, device=dev if dev is not None and dev.type == "cuda" else None)
    if not handoffs:
        return 0
    flat = torch.cat([t.reshape(-1) for h in handoffs for t in list(h.k) + list(h.v)])
    dist.send(flat, dst, group=group)
    return flat.numel() * flat.element_size()


def recv_handoffs(src: int, device, group=None) -> list[PrefillHandoff]:
    """Receive the hand-offs that `send_handoffs` sent from global rank `src`."""
    device = torch.device(device)
    box = [None]
    dist.recv_object_list(box, src=src, group=group, device=device if device.type == "cuda" else None)
    meta = box[0]
    if not meta:
        return []
    dtype = getattr(torch, meta[0][4].replace("torch.", ""))
    total = 0
    for _, _, _, shapes, _, _ in meta:
        for shp in shapes:
            n = 1
            for d in shp:
                n *= d
            total += 2 * n
    flat = torch.empty(total, dtype=dtype, device=device)
    dist.recv(flat, src, group=group)
    out, off = [], 0
    for req, tok, lp, shapes, _, ex in meta:
        ks, vs = [], []
        for dst_list in (ks, vs):
            for shp in shapes:
                n = 1
                for d in shp:
                    n *= d
                dst_list.append(flat[off:off + n].view(shp))
                off += n
        out.append(PrefillHandoff(req, ks, vs, tok, lp, ex))
    return out


_STEP_END = "__step_end__"


class RemotePrefill:
    """Decode-side stub of a paired prefill rank: `prefill(requests)` sends them and returns the
    hand-offs; `end_step()` tells the prefill rank that this rollout step has no more requests."""

    def __init__(self, peer: int, device, group=None):
        self.peer, self.device, self.group = peer, torch.device(device), group

    def prefill(self, reqs) -> list[PrefillHandoff]:
        dev = self.device if self.device.type == "cuda" else None
        dist.send_object_list([list(reqs)], dst=self.peer, group=self.group, device=dev)
        return recv_handoffs(self.peer, self.device, self.group)

    def end_step(self) -> None:
        dev = self.device if self.device.type == "cuda" else None
        dist.send_object_list([_STEP_END], dst=self.peer, group=self.group, device=dev)


def serve_prefill_step(engine, peer: int, group=None) -> int:
    """Prefill-rank loop of one rollout step: prefill every request batch the paired decode rank
    sends and return the hand-offs, until it ends the step. Returns the requests served."""
    dev = engine.dev if engine.dev.type == "cuda" else None
    served = 0
    while True:
        box = [None]
        dist.recv_object_list(box, src=peer, group=group, device=dev)
        msg = box[0]
        if isinstance(msg, str) and msg == _STEP_END:
            return served
        hs = engine.prefill_handoffs(msg) if msg else []
        send_handoffs(hs, peer, group)
        served += len(hs)
