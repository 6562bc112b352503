"""Speculative rollout with the model's multi-token-prediction (MTP) layer as the draft.

Per decode step and sequence (last token x_L at position L, not yet fed to the main model):

  1. draft: the MTP layer turns (main hidden of position L - 1, embedding of x_L) into a
     distribution q over x_{L+1} and proposes d ~ q. The MTP layer has its own paged K/V cache
     (one layer, same pages and slots as the main cache), filled for every position it has seen.
  2. verify: ONE main-model decode pass over two rows per sequence — (x_L, position L) and
     (d, position L + 1) — through the engine's paged cache: each layer writes both rows' K/V
     before its attention, and the paged decode kernel takes a context length per row, so the
     second row attends to the first. It yields p_L (over x_{L+1}) and p_{L+1} (over x_{L+2}).
  3. accept d with probability min(1, p_L(d) / q(d)) (greedy: when d is p_L's argmax); then
     x_{L+2} ~ p_{L+1}, two tokens for one pass. On rejection x_{L+1} ~ normalise(max(0, p_L - q))
     (greedy: argmax p_L), one token. Either way every emitted token is distributed exactly as
     under the main model alone (standard speculative sampling: Leviathan et al. 2023, Chen et
     al. 2023), and its recorded log-prob is the main model's log p at that position.

The stale K/V a rejected draft left at position L + 1 is overwritten when that position is fed.
The verify pass streams the weights once for up to two tokens, which is where the decode-bound
rollout gains. Eager host-driven loop (no CUDA graph), sampling with torch on the verify pass's
fp32 logits; standard softmax-attention models without tensor parallelism; no top-k / top-p
and no routed-expert recording on this path.

Reference role: SGLang speculative decoding with an MTP / NextN draft (EAGLE-style, enabled by
the --sglang-speculative-* flags in the reference's scripts; README "speculative rollout").
"""
from __future__ import annotations

import math
import time

import torch

from miles_b200.models.transformer import PAGE
from miles_b200.ops import gemm as G
from miles_b200.ops.attention import VarlenMeta


def _u01(seed: int, pos: int, tag: int, dev) -> float:
    """A uniform in [0, 1) keyed by (request seed, position, use): reproducible per request
    whatever the batch."""
    g = torch.Generator().manual_seed((seed * 1000003 + pos * 8191 + tag * 131) % (2 ** 63))
    return float(torch.rand(1, generator=g))


def _pick(probs: torch.Tensor, u: float) -> int:
    """Inverse-CDF draw from a probability row."""
    c = torch.cumsum(probs.double(), 0)
    v = torch.tensor([u * float(c[-1])], dtype=c.dtype, device=c.device)
    i = int(torch.searchsorted(c, v, right=True))  # first index whose CDF exceeds v
    return min(i, probs.numel() - 1)


class MTPSpeculativeDecoder:
    def __init__(self, engine):
        m = engine.model
        if not m.mtp_ids:
            raise ValueError("speculative decoding with an MTP draft needs a model with MTP layers "
                             "(mtp_num_layers > 0)")
        if m.gdn is not None or m.gattn is not None or m.mla is not None or m.tp is not None:
            raise ValueError("MTP speculative decoding supports standard softmax-attention models "
                             "without tensor parallelism")
        self.e, self.m = engine, m
        self.j = m.mtp_ids[0]
        self.kc = self.vc = None
        self.stats = {"spec_steps": 0, "spec_drafts": 0, "spec_accepted": 0}
        # tests: fn(request, position) -> the draft token at `position` (q is then one-hot)
        self.draft_override = None

    # ------------------------------------------------------------------ helpers
    def _ensure_cache(self):
        ref = self.e.cache.k[0]
        if self.kc is None or self.kc.shape != ref.shape:
            self.kc = torch.zeros_like(ref)
            self.vc = torch.zeros_like(ref)

    def _logits(self, y: torch.Tensor) -> torch.Tensor:
        return G.matmul_nt(y.contiguous(), self.m.lm_head_weight(), out_dtype=torch.float32)

    @staticmethod
    def _probs(z: torch.Tensor, inv_t: float) -> torch.Tensor:
        if inv_t <= 0:
            p = torch.zeros_like(z)
            p[int(z.argmax())] = 1.0
            return p
        return torch.softmax(z * inv_t, -1)

    @staticmethod
    def _lp(z: torch.Tensor, inv_t: float, tok: int) -> float:
        zz = z * (inv_t if inv_t > 0 else 1.0)
        return float(zz[tok] - torch.logsumexp(zz, -1))

    # ------------------------------------------------------------------ generate
    @torch.no_grad()
    def generate(self, reqs, stop_when=None, callbacks=None) -> list:
        """Same contract as RolloutEngine.generate: `stop_when(results)` is checked after every
        verify pass with the finished results so far (partial rollout: when it returns True the
        unfinished sequences return their tokens so far with finish_reason "abort", requests
        not started return empty); `callbacks` {rid: fn} receive their results as they finish
        instead of the returned list."""
        from miles_b200.engine.engine import GenResult

        e = self.e
        e.aborted = False
        self.stats = {"spec_steps": 0, "spec_drafts": 0, "spec_accepted": 0}  # this call's
        results: dict[int, GenResult] = {}
        cbs = dict(callbacks or {})

        def finish(res):
            cb = cbs.pop(res.rid, None)
            if cb is not None:
                cb(res)
            else:
                results[res.rid] = res

        def stop() -> bool:
            return e.aborted or (stop_when is not None and bool(stop_when(results)))

        e.resume_memory()
        self._ensure_cache()
        for r in reqs:
            if r.top_k > 0 or r.top_p < 1.0 or r.return_routed_experts:
                raise ValueError("speculative decoding: top-k / top-p / routed-expert recording "
                                 "are not supported on this path")
        t0 = time.perf_counter()
        pending = list(reqs)
        aborted = False
        while pending and not aborted:
            wave, rest, pages = [], [], []
            for r in pending:
                need = math.ceil((len(r.prompt) + r.max_new_tokens + 1) / PAGE)
                if need > e.max_pages_per_seq:
                    raise ValueError(f"request needs {need} pages > max_pages_per_seq")
                if not rest and len(wave) < e.max_batch and need <= len(e.free_pages):
                    wave.append(r)
                    pages.append([e.free_pages.pop() for _ in range(need)])
                else:
                    rest.append(r)
            if not wave:
                raise RuntimeError("speculative decoding: not enough KV pages for one request")
            try:
                aborted = self._run(wave, pages, finish, stop)
            finally:
                for pg in pages:
                    e.free_pages.extend(pg)
            pending = rest
        for r in pending:  # not started before the abort
            finish(GenResult(r.rid, [], [], "abort", None, self.m.weight_version, {"spec_decode": True}))
        e.stats.update(self.stats)
        e.stats["spec_time"] = time.perf_counter() - t0
        return [results[r.rid] for r in reqs if r.rid in results]

    def _run(self, wave, pages, finish, stop) -> bool:
        """Generate one admitted wave; finished sequences are reported through `finish` as they
        end. Returns True when `stop()` cut the wave short (the rest reported as "abort")."""
        from miles_b200.engine.engine import GenResult

        e, m, dev = self.e, self.m, self.e.dev
        B = len(wave)
        slot = lambda b, p: pages[b][p // PAGE] * PAGE + p % PAGE  # noqa: E731
        maxp = max(len(p) for p in pages)
        pt = torch.zeros(B, maxp, dtype=torch.int32)
        for b, p in enumerate(pages):
            pt[b, :len(p)] = torch.tensor(p, dtype=torch.int32)
        pt = pt.to(dev)
        inv_t = [1.0 / r.temperature if r.temperature > 0 else 0.0 for r in wave]

        # ---- main prefill, first token
        cu, toks, slots, pos = [0], [], [], []
        for b, r in enumerate(wave):
            toks.extend(r.prompt)
            slots.extend(slot(b, p) for p in range(len(r.prompt)))
            pos.extend(range(len(r.prompt)))
            cu.append(len(toks))
        meta = VarlenMeta(cu, dev)
        h = m.forward_prefill(torch.tensor(toks, dtype=torch.int32, device=dev), meta, e.cache,
                              torch.tensor(slots, dtype=torch.int64, device=dev))
        z = self._logits(h.index_select(0, torch.tensor([c - 1 for c in cu[1:]], device=dev)))
        seq = [list(r.prompt) for r in wave]
        gen = [[] for _ in wave]
        lps = [[] for _ in wave]
        done = [False] * B
        reason = ["length"] * B

        def emit(b, tok, lp):
            gen[b].append(tok)
            lps[b].append(lp)
            seq[b].append(tok)
            if tok in wave[b].stop_token_ids:
                done[b], reason[b] = True, "stop"
            elif len(gen[b]) >= wave[b].max_new_tokens:
                done[b], reason[b] = True, "length"

        reported = [False] * B

        def report():
            for b in range(B):
                if done[b] and not reported[b]:
                    reported[b] = True
                    finish(GenResult(wave[b].rid, gen[b], lps[b], reason[b], None, m.weight_version,
                                     {"spec_decode": True}))

        for b, r in enumerate(wave):
            L = len(r.prompt)
            tok = (int(z[b].argmax()) if inv_t[b] <= 0
                   else _pick(self._probs(z[b], inv_t[b]), _u01(r.seed, L, 0, dev)))
            emit(b, tok, self._lp(z[b], inv_t[b], tok))

        # ---- MTP prefill over every prompt position t (pair: h[t], token t + 1)
        nxt, mslots = [], []
        for b in range(B):
            nxt.extend(seq[b][1:len(wave[b].prompt) + 1])
            mslots.extend(slot(b, p) for p in range(len(wave[b].prompt)))
        _, ym = m.mtp_infer(self.j, h, torch.tensor(nxt, dtype=torch.int32, device=dev),
                            meta.positions, self.kc, self.vc,
                            torch.tensor(mslots, dtype=torch.int64, device=dev), meta=meta)
        q_last = self._logits(ym.index_select(0, torch.tensor([c - 1 for c in cu[1:]], device=dev)))

        # ---- decode loop
        while not all(done):
            live = [b for b in range(B) if not done[b]]
            # draft from the MTP distribution of the last fed pair
            drafts, qp = {}, {}
            for i, b in enumerate(live):
                L = len(seq[b]) - 1
                if self.draft_override is not None:
                    drafts[b] = int(self.draft_override(wave[b], L + 1))
                    qp[b] = torch.zeros_like(q_last[b])
                    qp[b][drafts[b]] = 1.0
                    continue
                qrow = self._probs(q_last[b], inv_t[b])
                drafts[b] = (int(q_last[b].argmax()) if inv_t[b] <= 0
                             else _pick(qrow, _u01(wave[b].seed, L + 1, 1, dev)))
                qp[b] = qrow
            # verify: rows (x_L, L) and (d, L + 1) per live sequence
            tk, ps, sl, cl, rows = [], [], [], [], []
            for b in live:
                L = len(seq[b]) - 1
                tk += [seq[b][L], drafts[b]]
                ps += [L, L + 1]
                sl += [slot(b, L), slot(b, L + 1)]
                cl += [L + 1, L + 2]
                rows += [b, b]
            pos_t = torch.tensor(ps, dtype=torch.int32, device=dev)
            hv = m.forward_decode(torch.tensor(tk, dtype=torch.int32, device=dev), pos_t, e.cache,
                                  pt.index_select(0, torch.tensor(rows, device=dev)).contiguous(),
                                  torch.tensor(cl, dtype=torch.int32, device=dev),
                                  torch.tensor(sl, dtype=torch.int64, device=dev))
            zv = self._logits(hv)
            self.stats["spec_steps"] += 1
            self.stats["spec_drafts"] += len(live)
            # accept / reject; collect the MTP pairs each sequence still has to feed
            m_h, m_tok, m_pos, m_slot, m_row, m_last = [], [], [], [], [], {}
            for i, b in enumerate(live):
                L = len(seq[b]) - 1
                zL, zL1 = zv[2 * i], zv[2 * i + 1]
                pL = self._probs(zL, inv_t[b])
                d = drafts[b]
                if inv_t[b] <= 0:
                    ok = int(zL.argmax()) == d
                else:
                    ok = _u01(wave[b].seed, L + 1, 2, dev) * float(qp[b][d]) < float(pL[d])
                if ok:
                    self.stats["spec_accepted"] += 1
                    emit(b, d, self._lp(zL, inv_t[b], d))
                    pairs = [(hv[2 * i], d, L)]
                    if not done[b]:
                        t2 = (int(zL1.argmax()) if inv_t[b] <= 0
                              else _pick(self._probs(zL1, inv_t[b]), _u01(wave[b].seed, L + 2, 0, dev)))
                        emit(b, t2, self._lp(zL1, inv_t[b], t2))
                        pairs.append((hv[2 * i + 1], t2, L + 1))
                else:
                    if inv_t[b] <= 0:
                        t1 = int(zL.argmax())
                    else:
                        res = (pL - qp[b]).clamp_min(0)
                        res = res if float(res.sum()) > 0 else pL
                        t1 = _pick(res, _u01(wave[b].seed, L + 1, 3, dev))
                    emit(b, t1, self._lp(zL, inv_t[b], t1))
                    pairs = [(hv[2 * i], t1, L)]
                if done[b]:
                    continue
                for hh, tok, p in pairs:
                    m_h.append(hh)
                    m_tok.append(tok)
                    m_pos.append(p)
                    m_slot.append(slot(b, p))
                    m_row.append(b)
                m_last[b] = len(m_h) - 1
            report()
            if not all(done) and stop():
                for b in range(B):
                    if not done[b]:
                        done[b], reason[b] = True, "abort"
                report()
                return True
            if not m_h:
                break
            _, ym = m.mtp_infer(self.j, torch.stack(m_h), torch.tensor(m_tok, dtype=torch.int32, device=dev),
                                torch.tensor(m_pos, dtype=torch.int32, device=dev), self.kc, self.vc,
                                torch.tensor(m_slot, dtype=torch.int64, device=dev),
                                page_table=pt.index_select(0, torch.tensor(m_row, device=dev)).contiguous(),
                                ctx_lens=torch.tensor([p + 1 for p in m_pos], dtype=torch.int32, device=dev))
            zq = self._logits(ym)
            q_last = {b: zq[k] for b, k in m_last.items()}
        report()
        return False
