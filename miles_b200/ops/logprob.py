"""Chunked LM-head log-prob / entropy and token sampling (csrc/rl_ops.cu + tcgen05 GEMM).

`lm_head_logprob(h, W, targets, temperature)` computes log softmax(h W^T / T)[target] and the
entropy per row without ever materialising the full [n, V] logits: rows are processed in chunks
whose fp32 logits live only inside the chunk (recomputed in backward). The rollout sampler
(`sample_from_hidden`) uses the same GEMM and the same row-statistics reduction, so the
log-prob of a sampled token equals the trainer's log-prob of that token bit for bit.

Reference roles replaced: ppo_utils.py get_log_probs_and_entropy / vocab-parallel CE
(:151-194, :659-717), `--log-probs-chunk-size`, SGLang sampler log-softmax (sglang.patch:500-523).
"""
from __future__ import annotations

import torch

from miles_b200.ops import gemm as G
from miles_b200.ops._lib import lib, use_native

DEFAULT_CHUNK = 4096


def logprob_ref(h, W, targets, temperature: float = 1.0):
    z = (h.float() @ W.float().t()) / temperature
    lsm = z.log_softmax(-1)
    lp = lsm.gather(1, targets.long()[:, None])[:, 0]
    ent = -(lsm.exp() * lsm).sum(-1)
    return lp, ent


class _LMHeadLogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, targets, inv_temp, chunk):
        n = h.shape[0]
        V = W.shape[0]
        dev = h.device
        h = h.contiguous()
        logp = torch.empty(n, dtype=torch.float32, device=dev)
        ent = torch.empty(n, dtype=torch.float32, device=dev)
        lse = torch.empty(n, dtype=torch.float32, device=dev)
        buf = torch.empty(min(chunk, max(n, 1)), V, dtype=torch.float32, device=dev)
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            z = buf[: e - s]
            G.matmul_nt(h[s:e], W, out=z)
            lib().logprob_fwd(z, targets[s:e], inv_temp, logp[s:e], ent[s:e], lse[s:e])
        del buf
        ctx.save_for_backward(h, W, targets, lse, ent)
        ctx.cfg = (inv_temp, chunk)
        return logp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):
        h, W, targets, lse, ent = ctx.saved_tensors
        inv_temp, chunk = ctx.cfg
        n, H = h.shape
        V = W.shape[0]
        dev = h.device
        dh = torch.empty_like(h)
        main = G.main_grad_of(W)
        dW = None
        if main is None and ctx.needs_input_grad[1]:
            dW = torch.zeros(V, H, dtype=torch.float32, device=dev)
        zbuf = torch.empty(min(chunk, max(n, 1)), V, dtype=torch.float32, device=dev)
        dbuf = torch.empty(min(chunk, max(n, 1)), V, dtype=torch.bfloat16, device=dev)
        g_lp = g_lp.contiguous() if g_lp is not None else None
        g_ent = g_ent.contiguous() if g_ent is not None else None
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            z = zbuf[: e - s]
            d = dbuf[: e - s]
            G.matmul_nt(h[s:e], W, out=z)
            lib().logprob_bwd(z, targets[s:e], inv_temp, lse[s:e],
                              None if g_lp is None else g_lp[s:e],
                              None if g_ent is None else g_ent[s:e], ent[s:e], d)
            G.matmul_nn(d, W, out=dh[s:e])
            if main is not None:
                G.matmul_tn(d, h[s:e], out=main, accumulate=True)
            elif dW is not None:
                G.matmul_tn(d, h[s:e], out=dW, accumulate=True)
        return dh, (dW.to(W.dtype) if dW is not None else None), None, None, None


def lm_head_logprob(h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor,
                    temperature: float = 1.0, chunk: int = DEFAULT_CHUNK):
    """h [n,H] bf16, W [V,H] bf16, targets int32 [n] -> (logp fp32 [n], entropy fp32 [n])."""
    if not use_native(h):
        return logprob_ref(h, W, targets, temperature)
    return _LMHeadLogProb.apply(h, W, targets.int().contiguous(), 1.0 / temperature, chunk)


def sampling_threshold(z: torch.Tensor, inv_temps: torch.Tensor, top_k: torch.Tensor | None,
                       top_p: torch.Tensor | None, k_max: int) -> torch.Tensor:
    """Per-row logit threshold of top-k / top-p sampling: tokens with z >= thr are kept.
    top_k int32 [B] (<= 0: off; at most k_max), top_p fp32 [B] (>= 1: off). The nucleus is the
    smallest prefix of the tokens sorted by probability (at the row's temperature) whose mass
    reaches top_p. Runs without host synchronisation (capturable in a CUDA graph)."""
    B = z.shape[0]
    thr = torch.full((B,), float("-inf"), dtype=torch.float32, device=z.device)
    if top_k is not None and k_max > 0:
        vals = torch.topk(z, k_max, dim=1).values                     # [B, k_max] descending
        k = top_k.long().clamp(1, k_max) - 1
        tk = vals.gather(1, k[:, None])[:, 0]
        thr = torch.where(top_k > 0, torch.maximum(thr, tk), thr)
    if top_p is not None:
        it = torch.where(inv_temps > 0, inv_temps, torch.ones_like(inv_temps))
        srt, _ = torch.sort(z, dim=1, descending=True)
        p = torch.softmax(srt * it[:, None], dim=1)
        before = torch.cumsum(p, dim=1) - p                              # mass of the better tokens
        n_keep = (before < top_p[:, None]).sum(1).clamp_min(1)
        tp = srt.gather(1, (n_keep - 1)[:, None])[:, 0]
        thr = torch.where(top_p < 1.0, torch.maximum(thr, tp), thr)
    return thr


def sample_from_hidden(h: torch.Tensor, W: torch.Tensor, inv_temps: torch.Tensor,
                       seeds: torch.Tensor, positions: torch.Tensor,
                       logits_buf: torch.Tensor | None = None, top_k: torch.Tensor | None = None,
                       top_p: torch.Tensor | None = None, k_max: int = 0):
    """Sample one token per row of h [B,H]. inv_temps fp32 [B] (<=0 => greedy), seeds int64 [B],
    positions int32 [B] (position of the sampled token); optional per-row top_k / top_p
    (see sampling_threshold). Returns (tokens int32, logp fp32): logp is the log-prob of the
    sampled token under the full temperature-scaled distribution (the trainer's log-prob)."""
    B = h.shape[0]
    V = W.shape[0]
    filt = top_k is not None or top_p is not None
    if not use_native(h):
        z = h.float() @ W.float().t()
        it = inv_temps.float()
        greedy = it <= 0
        zz = z * torch.where(greedy, torch.ones_like(it), it)[:, None]
        thr = sampling_threshold(z, it, top_k, top_p, k_max) if filt else None
        gen = torch.Generator(device=h.device)
        toks = []
        for b in range(B):
            row = zz[b] if thr is None else torch.where(z[b] >= thr[b], zz[b], torch.full_like(zz[b], float("-inf")))
            if bool(greedy[b]):
                toks.append(int(row.argmax()))
            else:
                gen.manual_seed(int(seeds[b]) * 1000003 + int(positions[b]))
                toks.append(int(torch.multinomial(row.softmax(-1), 1, generator=gen)))
        tok = torch.tensor(toks, dtype=torch.int32, device=h.device)
        lp = zz.log_softmax(-1).gather(1, tok.long()[:, None])[:, 0]
        return tok, lp
    z = logits_buf[:B] if logits_buf is not None else torch.empty(B, V, dtype=torch.float32, device=h.device)
    G.matmul_nt(h, W, out=z)
    tok = torch.empty(B, dtype=torch.int32, device=h.device)
    lp = torch.empty(B, dtype=torch.float32, device=h.device)
    thr = sampling_threshold(z, inv_temps, top_k, top_p, k_max).contiguous() if filt else None
    lib().sample(z, inv_temps, seeds, positions, tok, lp, thr)
    return tok, lp
