"""Causal GQA attention over packed variable-length sequences and paged-KV decode
(kernels in csrc/attention.cu). Head dim 128.

`varlen_attention(q, k, v, meta)` is differentiable (deterministic backward).
`decode_attention(q, k_cache, v_cache, page_table, ctx_lens)` is the rollout decode step; it
shares the forward's per-row block update, so a decode row is bitwise equal to the same row of
a training forward.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from miles_b200.ops._lib import err_word, lib, use_native

BLOCK = 64      # backward kernels: 64-row query blocks
FWD_TILE = 128  # forward kernel: 128-row query tiles
PAGE = 64  # KV-cache page size (tokens); equals the attention key block
CHUNK_PAGES = 16  # keys are merged in canonical 1024-key chunks (csrc/attention.cu)


def to_device(a: np.ndarray, device) -> torch.Tensor:
    """Host array -> device tensor through a pinned staging buffer with an asynchronous copy
    (a pageable source would make the copy wait for the stream, stalling the host)."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if torch.device(device).type != "cuda":
        return t.to(device)
    staged = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    staged.copy_(t)
    return staged.to(device, non_blocking=True)


def _block_table_np(cu: np.ndarray, rows: int) -> tuple[np.ndarray, np.ndarray]:
    lens = np.diff(cu)
    n = (lens + rows - 1) // rows
    seq = np.repeat(np.arange(len(lens), dtype=np.int32), n)
    starts = np.repeat(np.cumsum(n) - n, n)
    idx = (np.arange(int(n.sum())) - starts).astype(np.int32)
    order = np.argsort(-idx, kind="stable")
    return seq[order], idx[order]


def block_table(cu_seqlens: list[int], device, rows: int = 64) -> tuple[torch.Tensor, torch.Tensor]:
    """(seq index, block index) of every `rows`-row block of every sequence, longest-work first
    (64-row blocks for the backward kernels, 128-row tiles for the forward)."""
    seq, idx = _block_table_np(np.asarray(cu_seqlens, dtype=np.int64), rows)
    return to_device(seq, device), to_device(idx, device)


class VarlenMeta:
    """Host-built metadata of a packed batch (built once per micro-batch, reused by layers)."""

    def __init__(self, cu_seqlens: list[int], device):
        self.cu_list = [int(c) for c in cu_seqlens]
        cu = np.asarray(self.cu_list, dtype=np.int64)
        self.cu = to_device(cu.astype(np.int32), device)
        self.blk_seq, self.blk_idx = block_table(self.cu_list, device)
        self.tile_seq, self.tile_idx = block_table(self.cu_list, device, FWD_TILE)
        self.total = self.cu_list[-1]
        if len(cu) > 1:
            lens = np.diff(cu)
            pos = (np.arange(int(cu[-1]), dtype=np.int64) - np.repeat(cu[:-1], lens)).astype(np.int32)
        else:
            pos = np.zeros(0, dtype=np.int32)
        self.positions = to_device(pos, device)


def attention_ref(q, k, v, cu_seqlens: list[int], scale: float | None = None):
    """fp32 reference: causal softmax attention per sequence with GQA."""
    T, nq, D = q.shape
    nkv = k.shape[1]
    G = nq // nkv
    scale = scale or 1.0 / math.sqrt(D)
    out = torch.zeros(T, nq, D, dtype=torch.float32, device=q.device)
    for b in range(len(cu_seqlens) - 1):
        s, e = cu_seqlens[b], cu_seqlens[b + 1]
        if e == s:
            continue
        qq = q[s:e].float().transpose(0, 1)
        kk = k[s:e].float().repeat_interleave(G, 1).transpose(0, 1)
        vv = v[s:e].float().repeat_interleave(G, 1).transpose(0, 1)
        sc = qq @ kk.transpose(1, 2) * scale
        L = e - s
        mask = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
        sc = sc.masked_fill(mask, float("-inf"))
        out = out.index_copy(0, torch.arange(s, e, device=q.device), (sc.softmax(-1) @ vv).transpose(0, 1))
    return out


class _VarlenAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, meta: VarlenMeta, scale):
        T, nq, D = q.shape
        nkv = k.shape[1]
        o = torch.empty(T, nq, D, dtype=torch.bfloat16, device=q.device)
        lse = torch.empty(nq, T, dtype=torch.float32, device=q.device)
        q2, k2, v2 = q.reshape(T, nq * D), k.reshape(T, nkv * D), v.reshape(T, nkv * D)
        lib().attn_fwd(q2, k2, v2, o.view(T, nq * D), lse, meta.cu, meta.tile_seq, meta.tile_idx,
                       nq, nkv, scale, err_word(q.device))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.meta = meta
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        meta = ctx.meta
        T, nq, D = q.shape
        nkv = k.shape[1]
        do = do.contiguous()
        dq = torch.empty_like(q)
        dk = torch.empty_like(k)
        dv = torch.empty_like(v)
        delta = torch.empty(nq, T, dtype=torch.float32, device=q.device)
        lib().attn_bwd(q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1), o.view(T, -1),
                       do.view(T, -1), lse, delta, dq.view(T, -1), dk.view(T, -1), dv.view(T, -1),
                       meta.cu, meta.tile_seq, meta.tile_idx, nq, nkv, ctx.scale,
                       err_word(q.device))
        return dq, dk, dv, None, None


def varlen_attention(q, k, v, meta: VarlenMeta, scale: float | None = None):
    """q [T,nq,128], k/v [T,nkv,128] (bf16, contiguous) -> o [T,nq,128]."""
    scale = scale or 1.0 / math.sqrt(q.shape[-1])
    if not use_native(q):
        return attention_ref(q, k, v, meta.cu_list, scale).to(q.dtype)
    return _VarlenAttn.apply(q, k, v, meta, scale)


def decode_attention_ref(q, k_cache, v_cache, page_table, ctx_lens, scale=None):
    B, nq, D = q.shape
    nkv = k_cache.shape[1]
    G = nq // nkv
    scale = scale or 1.0 / math.sqrt(D)
    out = torch.empty_like(q)
    for b in range(B):
        L = int(ctx_lens[b])
        pages = page_table[b, : (L + PAGE - 1) // PAGE].long()
        slots = (pages[:, None] * PAGE + torch.arange(PAGE, device=q.device)[None]).reshape(-1)[:L]
        kk = k_cache[slots].float().repeat_interleave(G, 1).transpose(0, 1)
        vv = v_cache[slots].float().repeat_interleave(G, 1).transpose(0, 1)
        sc = (q[b].float()[:, None, :] @ kk.transpose(1, 2))[:, 0] * scale
        out[b] = (sc.softmax(-1)[:, None, :] @ vv)[:, 0].to(q.dtype)
    return out


def decode_attention(q, k_cache, v_cache, page_table, ctx_lens, scale: float | None = None,
                     out: torch.Tensor | None = None):
    """q [B,nq,128]; caches [num_slots, nkv, 128] (slot = page*64 + offset);
    page_table int32 [B, max_pages]; ctx_lens int32 [B] (keys incl. the current token)."""
    B, nq, D = q.shape
    nkv = k_cache.shape[1]
    scale = scale or 1.0 / math.sqrt(D)
    if not use_native(q):
        r = decode_attention_ref(q, k_cache, v_cache, page_table, ctx_lens, scale)
        if out is not None:
            out.copy_(r)
            return out
        return r
    if out is None:
        out = torch.empty_like(q)
    # keys are processed in 1024-key chunks merged in a fixed order (the same chunking the
    # training kernel uses); long contexts split across CTAs and need a small fp32 workspace
    nsplit = (page_table.shape[1] + CHUNK_PAGES - 1) // CHUNK_PAGES
    ws_o = ws_ml = None
    if nsplit > 1:
        ws_o = torch.empty(B * nq * nsplit * D, dtype=torch.float32, device=q.device)
        ws_ml = torch.empty(B * nq * nsplit * 2, dtype=torch.float32, device=q.device)
    lib().attn_decode(q, k_cache, v_cache, out, page_table, ctx_lens, nq, nkv, scale, ws_o, ws_ml,
                      err_word(q.device))
    return out
