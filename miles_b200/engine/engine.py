"""In-process rollout engine: paged KV cache, packed prefill, CUDA-graph decode.

The engine runs in the trainer's own process on the same GPU and reads the trainer's parameters
directly (colocated refit = bump the weight version; no copy), so there is no HTTP or IPC on the
hot path. A generation call:

  1. reserves ceil((prompt + max_new) / 64) KV pages per request (requests that do not fit wait
     for the next wave),
  2. prefills all prompts of the wave as one packed varlen batch and samples the first token,
  3. decodes one token per live sequence per step; each step is a captured CUDA graph for the
     smallest batch bucket >= live sequences (graphs are captured lazily per bucket),
  4. records per-token log-probs (bitwise equal to the trainer's) and, for MoE models, the
     routed experts of every token (Rollout Routing Replay).

Reference roles replaced: the SGLang engine + server (backends/sglang_utils/sglang_engine.py,
sglang.patch routed-experts capture :308-378, sampler log-softmax :500-523) and the
torch_memory_saver release/resume of KV memory (E15).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from miles_b200.models.transformer import KVCache, Transformer
from miles_b200.ops.attention import PAGE, VarlenMeta
from miles_b200.ops import _lib
from miles_b200.ops.logprob import sample_from_hidden

_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256, 384, 512)


@dataclass
class GenRequest:
    prompt: list[int]
    max_new_tokens: int
    temperature: float = 1.0
    seed: int = 0
    stop_token_ids: tuple = ()
    return_routed_experts: bool = False
    rid: int = 0


@dataclass
class GenResult:
    rid: int
    tokens: list[int]
    logprobs: list[float]
    finish_reason: str                     # "stop" | "length" | "abort"
    routed_experts: np.ndarray | None = None  # [prompt+resp-1, L_moe, k] int32
    weight_version: int = 0
    meta: dict = field(default_factory=dict)


class _Seq:
    __slots__ = ("req", "pages", "out", "lps", "pos", "done", "reason", "experts", "wave_idx")

    def __init__(self, req: GenRequest, pages: list[int]):
        self.req = req
        self.pages = pages
        self.out: list[int] = []
        self.lps: list[float] = []
        self.pos = len(req.prompt)  # position of the next token to be written
        self.done = False
        self.reason = ""
        self.experts: list[np.ndarray] = []
        self.wave_idx = 0  # row of this sequence in the linear-attention state cache


class RolloutEngine:
    def __init__(self, model: Transformer, max_batch: int = 64, num_pages: int | None = None,
                 mem_fraction: float = 0.9, use_cuda_graph: bool = True, max_pages_per_seq: int = 160):
        self.model = model
        self.cfg = model.cfg
        self.dev = model.device
        self.max_batch = max_batch
        self.use_graph = use_cuda_graph and self.dev.type == "cuda"
        self.max_pages_per_seq = max_pages_per_seq
        self._num_pages_req = num_pages
        self._mem_fraction = mem_fraction
        self.cache: KVCache | None = None
        self.graphs: dict[int, tuple] = {}
        self.graph_launches: dict[int, int] = {}
        self.pool = None
        self.aborted = False
        self.stats = {}
        self.n_moe = sum(1 for i in range(self.cfg.num_layers) if self.cfg.layer_is_moe(i))

    # ------------------------------------------------------------------ memory
    def kv_bytes_per_page(self) -> int:
        c = self.cfg
        from miles_b200.models.transformer import kv_cache_shape

        nkv, hd = kv_cache_shape(c, self.model.tp_size)
        return (1 if c.kv_lora_rank else 2) * c.num_layers * PAGE * nkv * hd * 2

    def resume_memory(self):
        """Allocate the KV cache (and lazily the decode graphs). Mirrors resume_memory_occupation."""
        if self.cache is not None:
            return
        n = self._num_pages_req
        if n is None:
            if self.dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(self.dev)
                n = int(free * self._mem_fraction) // self.kv_bytes_per_page()
            else:
                n = 1024
        n = max(n, 2)
        self.cache = KVCache(self.cfg, n, self.dev, self.model.dtype, self.model.tp_size,
                             max_seqs=self.max_batch + 1)
        self.free_pages = list(range(n - 1, 0, -1))  # page 0 = trash page for padded rows

    def release_memory(self):
        """Free KV cache and graphs (mirrors release_memory_occupation(kv_cache, cuda_graph))."""
        self.graphs.clear()
        self.pool = None
        self.cache = None
        if self.dev.type == "cuda":
            torch.cuda.empty_cache()

    # ------------------------------------------------------------------ graph machinery
    def _bucket(self, b: int) -> int:
        for s in _BUCKETS:
            if s >= b:
                return min(s, max(self.max_batch, b))
        return b

    def _static(self, B: int):
        dev = self.dev
        return {
            "tokens": torch.zeros(B, dtype=torch.int32, device=dev),
            "positions": torch.zeros(B, dtype=torch.int32, device=dev),
            "ctx": torch.ones(B, dtype=torch.int32, device=dev),
            "slots": torch.zeros(B, dtype=torch.int64, device=dev),
            "pt": torch.zeros(B, self.max_pages_per_seq, dtype=torch.int32, device=dev),
            "inv_t": torch.ones(B, dtype=torch.float32, device=dev),
            "seeds": torch.zeros(B, dtype=torch.int64, device=dev),
            "experts": torch.zeros(B, max(self.n_moe, 1), max(self.cfg.topk, 1), dtype=torch.int32, device=dev),
            # linear-attention state row of every batch row (padding rows: the spare last row)
            "state_rows": torch.full((B,), self.max_batch, dtype=torch.int64, device=dev),
        }

    def _step_fn(self, st):
        rec = []
        h = self.model.forward_decode(st["tokens"], st["positions"], self.cache, st["pt"], st["ctx"],
                                      st["slots"], record=rec if self.n_moe else None,
                                      state_rows=st["state_rows"])
        for j, idx in enumerate(rec):
            st["experts"][:, j].copy_(idx)
        # the sampled token sits at position `positions + 1`
        tok, lp = sample_from_hidden(h, self.model.lm_head_weight(), st["inv_t"], st["seeds"],
                                     st["positions"] + 1)
        return tok, lp

    def _get_step(self, B: int):
        if B in self.graphs:
            return self.graphs[B]
        st = self._static(B)
        if not self.use_graph:
            entry = (None, st, None)
            self.graphs[B] = entry
            return entry
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step_fn(st)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        g = torch.cuda.CUDAGraph()
        n0 = _lib.launch_count()
        with torch.cuda.graph(g, pool=self.pool):
            out = self._step_fn(st)
        self.graph_launches[B] = _lib.launch_count() - n0
        entry = (g, st, out)
        self.graphs[B] = entry
        return entry

    # ------------------------------------------------------------------ generation
    def abort(self):
        self.aborted = True

    def generate(self, reqs: list[GenRequest]) -> list[GenResult]:
        """Continuous batching: requests are admitted whenever a batch slot and enough KV pages
        are free (prefilled as a packed batch, then joined to the running decode batch), and
        leave the batch as soon as they finish."""
        self.resume_memory()
        self.aborted = False
        results: dict[int, GenResult] = {}
        pending = list(reqs)
        live: list[_Seq] = []
        free_rows = list(range(self.max_batch - 1, -1, -1))  # linear-attention state rows
        t0 = time.perf_counter()
        n_decode_steps = n_prefills = 0
        while (pending or live) and not self.aborted:
            if pending and len(live) < self.max_batch:
                new, pending = self._admit(pending, self.max_batch - len(live))
                if new:
                    for sq in new:
                        sq.wave_idx = free_rows.pop()
                    self._prefill(new)
                    n_prefills += 1
                    live += new
                elif not live:
                    raise RuntimeError("KV cache too small for a single request")
            running = [sq for sq in live if not sq.done]
            if running:
                self._decode_step(running)
                n_decode_steps += 1
            still = []
            for sq in live:
                if sq.done:
                    results[sq.req.rid] = self._result(sq)
                    self.free_pages.extend(sq.pages)
                    free_rows.append(sq.wave_idx)
                else:
                    still.append(sq)
            live = still
        if self.aborted:
            for sq in live:
                sq.done, sq.reason = True, "abort"
                results[sq.req.rid] = self._result(sq)
                self.free_pages.extend(sq.pages)
            for r in pending:
                results[r.rid] = GenResult(r.rid, [], [], "abort", None, self.model.weight_version)
        self.stats = {"wall_s": time.perf_counter() - t0, "decode_steps": n_decode_steps,
                      "prefills": n_prefills}
        return [results[r.rid] for r in reqs]

    def _admit(self, pending, room: int):
        """Take requests in order while batch slots (`room`) and KV pages last."""
        wave, rest = [], []
        for r in pending:
            need = math.ceil((len(r.prompt) + r.max_new_tokens) / PAGE)
            if need > self.max_pages_per_seq:
                raise ValueError(f"request needs {need} pages > max_pages_per_seq")
            if not rest and len(wave) < room and need <= len(self.free_pages):
                wave.append(_Seq(r, [self.free_pages.pop() for _ in range(need)]))
            else:
                rest.append(r)  # keep arrival order: no request overtakes an earlier one
        return wave, rest

    def _slot(self, s: _Seq, pos: int) -> int:
        return s.pages[pos // PAGE] * PAGE + pos % PAGE

    def _prefill(self, wave: list[_Seq]) -> None:
        """Packed prefill of newly admitted sequences; samples and accepts their first token."""
        dev = self.dev
        cu = [0]
        toks, slots = [], []
        for s in wave:
            toks.extend(s.req.prompt)
            slots.extend(self._slot(s, p) for p in range(len(s.req.prompt)))
            cu.append(len(toks))
        meta = VarlenMeta(cu, dev)
        rec = [] if self.n_moe else None
        nvtx = dev.type == "cuda"
        if nvtx:
            torch.cuda.nvtx.range_push("prefill")
        h = self.model.forward_prefill(torch.tensor(toks, dtype=torch.int32, device=dev), meta,
                                       self.cache, torch.tensor(slots, dtype=torch.int64, device=dev),
                                       record=rec,
                                       state_rows=torch.tensor([s.wave_idx for s in wave],
                                                               dtype=torch.int64, device=dev))
        last = torch.tensor([c - 1 for c in cu[1:]], dtype=torch.long, device=dev)
        inv_t = torch.tensor([1.0 / s.req.temperature if s.req.temperature > 0 else 0.0 for s in wave],
                             dtype=torch.float32, device=dev)
        seeds = torch.tensor([s.req.seed for s in wave], dtype=torch.int64, device=dev)
        posn = torch.tensor([len(s.req.prompt) for s in wave], dtype=torch.int32, device=dev)
        tok, lp = sample_from_hidden(h.index_select(0, last).contiguous(), self.model.lm_head_weight(),
                                     inv_t, seeds, posn)
        if rec:
            ex = torch.stack(rec, 1).cpu().numpy()  # [T, L_moe, k]
            for b, s in enumerate(wave):
                if s.req.return_routed_experts:
                    s.experts.append(ex[cu[b]:cu[b + 1]])
        self._accept(wave, tok.tolist(), lp.tolist())
        if nvtx:
            torch.cuda.nvtx.range_pop()

    def _decode_step(self, live: list[_Seq]) -> None:
        """One token for every running sequence (CUDA graph of the batch bucket)."""
        nvtx = self.dev.type == "cuda"
        Bb = self._bucket(len(live))
        g, st, out = self._get_step(Bb)
        n = len(live)
        tokens = np.zeros(Bb, np.int32)
        pos = np.zeros(Bb, np.int32)
        ctx = np.ones(Bb, np.int32)
        slot = np.arange(Bb, dtype=np.int64) % PAGE  # trash page 0 for padding rows
        pt = np.zeros((Bb, self.max_pages_per_seq), np.int32)
        invt = np.ones(Bb, np.float32)
        seed = np.zeros(Bb, np.int64)
        srow = np.full(Bb, self.max_batch, np.int64)
        for j, s in enumerate(live):
            srow[j] = s.wave_idx
            p = len(s.req.prompt) + len(s.out) - 1  # position of the token being fed
            tokens[j] = s.out[-1]
            pos[j] = p
            ctx[j] = p + 1
            slot[j] = self._slot(s, p)
            pt[j, :len(s.pages)] = s.pages
            invt[j] = 1.0 / s.req.temperature if s.req.temperature > 0 else 0.0
            seed[j] = s.req.seed
        st["tokens"].copy_(torch.from_numpy(tokens), non_blocking=True)
        st["positions"].copy_(torch.from_numpy(pos), non_blocking=True)
        st["ctx"].copy_(torch.from_numpy(ctx), non_blocking=True)
        st["slots"].copy_(torch.from_numpy(slot), non_blocking=True)
        st["pt"].copy_(torch.from_numpy(pt), non_blocking=True)
        st["inv_t"].copy_(torch.from_numpy(invt), non_blocking=True)
        st["seeds"].copy_(torch.from_numpy(seed), non_blocking=True)
        st["state_rows"].copy_(torch.from_numpy(srow), non_blocking=True)
        if nvtx:
            torch.cuda.nvtx.range_push("decode_step")
        if g is not None:
            g.replay()
            _lib.add_launches(self.graph_launches[Bb])
            tok, lp = out
        else:
            tok, lp = self._step_fn(st)
        if self.n_moe and any(s.req.return_routed_experts for s in live):
            ex = st["experts"][:n].cpu().numpy().copy()
            for j, s in enumerate(live):
                if s.req.return_routed_experts:
                    s.experts.append(ex[j:j + 1])
        self._accept(live, tok[:n].tolist(), lp[:n].tolist())
        if nvtx:
            torch.cuda.nvtx.range_pop()

    def _accept(self, seqs, toks, lps):
        for s, t, l in zip(seqs, toks, lps):
            s.out.append(int(t))
            s.lps.append(float(l))
            if int(t) in s.req.stop_token_ids:
                s.done, s.reason = True, "stop"
            elif len(s.out) >= s.req.max_new_tokens:
                s.done, s.reason = True, "length"

    def _result(self, s: _Seq) -> GenResult:
        ex = None
        if s.req.return_routed_experts and s.experts:
            ex = np.concatenate(s.experts, 0)
            ex = ex[: len(s.req.prompt) + len(s.out) - 1]
        return GenResult(s.req.rid, s.out, s.lps, s.reason, ex, self.model.weight_version)
