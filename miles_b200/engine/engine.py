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

import dataclasses
import math
import threading
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
    top_k: int = 0          # <= 0: off
    top_p: float = 1.0      # >= 1: off


@dataclass
class GenResult:
    rid: int
    tokens: list[int]
    logprobs: list[float]
    finish_reason: str                     # "stop" | "length" | "abort"
    routed_experts: np.ndarray | None = None  # [prompt+resp-1, L_moe, k] int32
    weight_version: int = 0
    meta: dict = field(default_factory=dict)


@dataclass
class PrefillHandoff:
    """A request prefilled by a prefill engine, on its way to a decode engine (prefill / decode
    disaggregation): the prompt's K/V cache rows of every attention layer, the first sampled
    token with its log-prob, and the prompt's routing (R3)."""
    req: GenRequest
    k: list                       # per attention layer: [P, nkv, head_dim]
    v: list
    token: int
    logprob: float
    experts: np.ndarray | None = None  # [P, L_moe, k] uint8

    @property
    def rid(self):
        return self.req.rid

    @property
    def prompt(self):
        return self.req.prompt

    @property
    def max_new_tokens(self):
        return self.req.max_new_tokens

    @property
    def return_routed_experts(self):
        return self.req.return_routed_experts


class _Seq:
    __slots__ = ("req", "pages", "slot", "done", "reason", "prompt_experts", "order", "handoff")
    _count = 0

    def __init__(self, req: GenRequest, pages: list[int]):
        self.req = req
        self.pages = pages
        _Seq._count += 1
        self.order = _Seq._count  # admission order (the latest admitted is preempted first)
        self.handoff = None
        self.slot = -1           # sequence slot: row of the device decode state (and GDN state)
        self.done = False
        self.reason = ""


_NSTOP = 4  # stop token ids kept per sequence on the device


class DecodeState:
    """Per-slot decode state on the device (slots 0..S-1, slot S = spare for padding rows).

    s_tok: last sampled token (next step's input); s_pos: its position; s_done: frozen flag;
    s_nout / s_maxnew: generated / allowed tokens; s_pt: page-table row; s_invt, s_seed:
    sampling parameters; s_stop: up to 4 stop ids (-1 = none); s_rec: record routed experts.
    out_tok / out_lp [S+1, max_new]: generated tokens and their log-probs; out_exp
    [S+1, max_len, n_moe, k] uint8 (allocated on first use): routed experts of every fed
    position (prompt rows written at prefill)."""

    def __init__(self, S: int, max_pages: int, n_moe: int, topk: int, dev):
        i32 = dict(dtype=torch.int32, device=dev)
        self.S = S
        self.max_len = max_pages * PAGE
        self.s_tok = torch.zeros(S + 1, **i32)
        self.s_pos = torch.zeros(S + 1, **i32)
        self.s_done = torch.ones(S + 1, **i32)
        self.s_nout = torch.zeros(S + 1, **i32)
        self.s_maxnew = torch.zeros(S + 1, **i32)
        self.s_pt = torch.zeros(S + 1, max_pages, **i32)
        self.s_invt = torch.ones(S + 1, dtype=torch.float32, device=dev)
        self.s_seed = torch.zeros(S + 1, dtype=torch.int64, device=dev)
        self.s_stop = torch.full((S + 1, _NSTOP), -1, **i32)
        self.s_rec = torch.zeros(S + 1, **i32)
        self.s_topk = torch.zeros(S + 1, **i32)
        self.s_topp = torch.ones(S + 1, dtype=torch.float32, device=dev)
        self.out_tok = torch.zeros(S + 1, self.max_len, **i32)
        self.out_lp = torch.zeros(S + 1, self.max_len, dtype=torch.float32, device=dev)
        self.n_moe, self.topk = n_moe, topk
        self.out_exp: torch.Tensor | None = None
        self.dev = dev
        self.host_flags = (torch.zeros(2, S + 1, dtype=torch.int32).pin_memory()
                           if dev.type == "cuda" else torch.zeros(2, S + 1, dtype=torch.int32))

    def ensure_exp(self):
        if self.out_exp is None and self.n_moe:
            self.out_exp = torch.zeros(self.S + 1, self.max_len, self.n_moe, self.topk,
                                       dtype=torch.uint8, device=self.dev)
        return self.out_exp


def _prep_ref(ds: DecodeState, st: dict):
    """PyTorch form of csrc/engine_step.cu decode_prep (CPU path)."""
    rows = st["rows"].long()
    live = (rows != ds.S) & (ds.s_done[rows] == 0)
    p = torch.where(live, ds.s_pos[rows], torch.zeros_like(rows, dtype=torch.int32))
    live = live & (p > 0) & ((p // PAGE) < ds.s_pt.shape[1])
    p = torch.where(live, p, torch.zeros_like(p))
    pt = torch.where(live[:, None], ds.s_pt[rows], torch.zeros_like(ds.s_pt[rows]))
    st["pt"].copy_(pt)
    st["tokens"].copy_(torch.where(live, ds.s_tok[rows], torch.zeros_like(p)))
    st["positions"].copy_(p)
    st["ctx"].copy_(p + 1)
    j = torch.arange(rows.numel(), device=rows.device)
    page = pt.gather(1, (p // PAGE).long()[:, None])[:, 0].long()
    st["slots"].copy_(torch.where(live, page * PAGE + (p % PAGE).long(), j % PAGE))
    st["inv_t"].copy_(torch.where(live, ds.s_invt[rows], torch.ones_like(ds.s_invt[rows])))
    st["seeds"].copy_(torch.where(live, ds.s_seed[rows], torch.zeros_like(ds.s_seed[rows])))
    st["state_rows"].copy_(torch.where(live, rows, torch.full_like(rows, ds.S)))


def _commit_ref(ds: DecodeState, st: dict, tok, lp, experts):
    """PyTorch form of csrc/engine_step.cu decode_commit (CPU path)."""
    rows = st["rows"].long()
    live = (rows != ds.S) & (ds.s_done[rows] == 0) & (ds.s_pos[rows] > 0)
    r = rows[live]
    if r.numel() == 0:
        return
    t = tok[live].int()
    n = ds.s_nout[r].long()
    p = ds.s_pos[r].long()
    if experts is not None and ds.out_exp is not None:
        rec = (ds.s_rec[r] != 0) & (p < ds.max_len)
        ds.out_exp[r[rec], p[rec]] = experts.permute(1, 0, 2)[live][rec].to(torch.uint8)
    ok = n < ds.max_len
    ds.out_tok[r[ok], n[ok]] = t[ok]
    ds.out_lp[r[ok], n[ok]] = lp[live][ok].float()
    stop = (n + 1 >= ds.s_maxnew[r].long()) | (n + 1 >= ds.max_len)
    stop = stop | (ds.s_stop[r] == t[:, None]).any(1)
    ds.s_nout[r] = (n + 1).int()
    ds.s_tok[r] = t
    ds.s_pos[r] = (p + 1).int()
    ds.s_done[r] = torch.where(stop, torch.ones_like(t), ds.s_done[r])


class RolloutEngine:
    def __init__(self, model: Transformer, max_batch: int = 64, num_pages: int | None = None,
                 mem_fraction: float = 0.9, use_cuda_graph: bool = True, max_pages_per_seq: int = 160,
                 steps_per_sync: int = 8, persistent_kv: bool = True, prefill_tokens: int = 32768,
                 lazy_pages: bool = True, speculative: str | None = None):
        self.model = model
        self.cfg = model.cfg
        self.dev = model.device
        self.max_batch = max_batch
        self.use_graph = use_cuda_graph and self.dev.type == "cuda"
        self.max_pages_per_seq = max_pages_per_seq
        # decode steps run back to back on the device between two host visits (one graph)
        self.steps_per_sync = max(1, steps_per_sync)
        self.prefill_tokens = prefill_tokens   # token budget of one packed prefill
        # KV pages on demand: a sequence holds pages for its prompt and the next host visit's
        # decode steps only, and gets more as it grows; when the pool runs dry the latest
        # admitted sequence is preempted (its tokens kept, resumed later by re-prefill).
        # Otherwise every request reserves pages for prompt + max_new_tokens at admission.
        self.lazy_pages = lazy_pages
        self._num_pages_req = num_pages
        self._mem_fraction = mem_fraction
        self.cache: KVCache | None = None
        self.ds: DecodeState | None = None
        self.graphs: dict[int, tuple] = {}
        self.graph_launches: dict[int, int] = {}
        self.pool = None
        self.aborted = False
        self.dead = False            # set by a failed health check / injected crash
        self._lock = threading.Lock()
        self._inbox: list = []       # (GenRequest, callback) submitted while generate() runs
        self._serving = False
        self.stats = {}
        self.n_moe = sum(1 for i in range(self.cfg.num_layers) if self.cfg.layer_is_moe(i))
        self.native = _lib.use_native(torch.empty(0, device=self.dev))
        self._filt = (0, False)      # sampler restriction of the running batch (graph variant)
        # fixed-address KV cache: graphs survive release / resume (GPU only)
        self.use_arena = persistent_kv and self.use_graph and self.native
        self.arena = None
        self._arena_pages = 0
        self._num_pages = 0
        self._free_pages: list[int] | None = None
        # speculative rollout with the model's MTP layer as the draft (engine/speculative.py)
        self.speculative = None
        if speculative:
            self.enable_speculative(speculative)

    def enable_speculative(self, algo: str = "mtp"):
        """Route `generate` through speculative decoding: "mtp" (aliases "nextn", "eagle") drafts
        one token per step with the model's first MTP layer and verifies it in one main-model
        decode pass (engine/speculative.py)."""
        if str(algo).lower() not in ("mtp", "nextn", "eagle"):
            raise ValueError(f"unknown speculative algorithm {algo!r}")
        from miles_b200.engine.speculative import MTPSpeculativeDecoder

        self.speculative = MTPSpeculativeDecoder(self)

    # ------------------------------------------------------------------ memory
    def kv_bytes_per_page(self) -> int:
        c = self.cfg
        from miles_b200.models.transformer import kv_cache_shape

        nkv, hd = kv_cache_shape(c, self.model.tp_size)
        return (1 if c.kv_lora_rank else 2) * c.num_layers * PAGE * nkv * hd * 2

    def resume_memory(self):
        """Allocate the KV cache and the decode state (graphs are captured lazily). Mirrors
        resume_memory_occupation. On GPUs the cache lives in a fixed-address arena
        (engine/arena.py): after the first call, resuming maps fresh memory at the same
        addresses, so decode graphs captured earlier stay valid."""
        if self.cache is not None:
            return
        if self.ds is None:
            self.ds = DecodeState(self.max_batch, self.max_pages_per_seq, self.n_moe,
                                  max(self.cfg.topk, 1), self.dev)
        kw = dict(dtype=self.model.dtype, tp_size=self.model.tp_size, max_seqs=self.max_batch + 1)
        if self.arena is not None:
            self.cache = KVCache(self.cfg, self._arena_pages, self.dev, buffer=self.arena.map(), **kw)
            return
        n = self._num_pages_req
        if n is None:
            if self.dev.type == "cuda":
                free, _ = torch.cuda.mem_get_info(self.dev)
                # the routed-expert record buffer is allocated on first use: leave room for it
                reserve = (self.max_batch + 1) * self.ds.max_len * self.n_moe * max(self.cfg.topk, 1)
                # headroom for prefill activations and the decode graphs' memory pool
                headroom = 8 << 30
                n = int(max(free - reserve - headroom, 0) * self._mem_fraction) // self.kv_bytes_per_page()
            else:
                n = 1024
        n = max(n, 2)
        if self.use_arena:
            from miles_b200.engine.arena import DeviceArena

            self.arena = DeviceArena(KVCache.required_bytes(self.cfg, n, **kw), self.dev)
            self._arena_pages = n
            self.cache = KVCache(self.cfg, n, self.dev, buffer=self.arena.map(), **kw)
        else:
            self.cache = KVCache(self.cfg, n, self.dev, **kw)
        self._num_pages = n

    @property
    def free_pages(self) -> list[int]:
        if self._free_pages is None:
            self._free_pages = list(range(self._num_pages - 1, 0, -1))  # page 0 = trash page
        return self._free_pages

    def release_memory(self, levels=("kv_cache",)):
        """Free the engine's memory (mirrors release_memory_occupation with the reference's
        --offload-rollout-level tags). "kv_cache": the KV cache (with the arena its physical
        memory is unmapped and the addresses kept); "cuda_graph": the decode graphs, their
        memory pool and the decode state too (they are re-captured on the next rollout;
        without this tag they stay, since the arena keeps their addresses valid). "weight" has
        nothing to free: the colocated engine reads the trainer's parameter buffer."""
        levels = set(levels or ())
        self.cache = None
        self._free_pages = None
        drop_graphs = "cuda_graph" in levels or self.arena is None
        if self.arena is not None:
            self.arena.unmap()
        if drop_graphs:
            self.graphs.clear()
            self.graph_launches.clear()
            self.pool = None
            self.ds = None
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
            "rows": torch.full((B,), self.max_batch, dtype=torch.int32, device=dev),
            "tokens": torch.zeros(B, dtype=torch.int32, device=dev),
            "positions": torch.zeros(B, dtype=torch.int32, device=dev),
            "ctx": torch.ones(B, dtype=torch.int32, device=dev),
            "slots": torch.zeros(B, dtype=torch.int64, device=dev),
            "pt": torch.zeros(B, self.max_pages_per_seq, dtype=torch.int32, device=dev),
            "inv_t": torch.ones(B, dtype=torch.float32, device=dev),
            "seeds": torch.zeros(B, dtype=torch.int64, device=dev),
            # routing of each batch row, layer-major [L_moe, B, k] (each layer's slice contiguous)
            "experts": torch.zeros(max(self.n_moe, 1), B, max(self.cfg.topk, 1), dtype=torch.int32, device=dev),
            # linear-attention state row of every batch row (= its slot; padding: the spare row)
            "state_rows": torch.full((B,), self.max_batch, dtype=torch.int64, device=dev),
        }

    def _step_fn(self, st):
        """One decode step of the bucket: gather inputs from the slots, forward, sample, commit."""
        ds = self.ds
        rec_on = self.n_moe and ds.out_exp is not None
        if self.native:
            _lib.lib().decode_prep(st["rows"], ds.S, ds.s_tok, ds.s_pos, ds.s_done, ds.s_pt,
                                   ds.s_invt, ds.s_seed, st["tokens"], st["positions"], st["ctx"],
                                   st["slots"], st["pt"], st["inv_t"], st["seeds"],
                                   st["state_rows"], ds.S)
        else:
            _prep_ref(ds, st)
        h = self.model.forward_decode(st["tokens"], st["positions"], self.cache, st["pt"], st["ctx"],
                                      st["slots"], record=st["experts"] if rec_on else None,
                                      state_rows=st["state_rows"])
        # the sampled token sits at position `positions + 1`
        kmax, use_p = self._filt
        rows = st["rows"].long()
        tok, lp = sample_from_hidden(h, self.model.lm_head_weight(), st["inv_t"], st["seeds"],
                                     st["positions"] + 1,
                                     top_k=ds.s_topk[rows] if kmax else None,
                                     top_p=ds.s_topp[rows] if use_p else None, k_max=kmax)
        if self.native:
            _lib.lib().decode_commit(st["rows"], ds.S, tok, lp, st["experts"] if rec_on else None,
                                     ds.s_tok, ds.s_pos, ds.s_done, ds.s_nout, ds.s_maxnew,
                                     ds.s_stop, ds.out_tok, ds.out_lp,
                                     ds.out_exp if rec_on else None, ds.s_rec)
        else:
            _commit_ref(ds, st, tok, lp, st["experts"] if rec_on else None)

    def _get_steps(self, B: int):
        """(graph or None, static inputs) running `steps_per_sync` decode steps of bucket B."""
        key = (B, self.ds.out_exp is not None) + self._filt
        if key in self.graphs:
            return self.graphs[key]
        st = self._static(B)
        if not self.use_graph:
            entry = (None, st)
            self.graphs[key] = entry
            return entry
        # warm-up on a side stream with every row padding (writes only the trash page)
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
            for _ in range(self.steps_per_sync):
                self._step_fn(st)
        self.graph_launches[key] = _lib.launch_count() - n0
        entry = (g, st)
        self.graphs[key] = entry
        return entry

    # ------------------------------------------------------------------ generation
    def abort(self):
        self.aborted = True

    def submit(self, items: list) -> bool:
        """Hand [(GenRequest, callback(GenResult))] to a generate() call that is running in
        another thread: they join its batch at its next host visit (continuous batching across
        callers). Returns False when no call is running (the caller starts one)."""
        with self._lock:
            if not self._serving:
                return False
            self._inbox.extend(items)
            return True

    def health_check(self) -> bool:
        """Liveness probe: not marked dead, and no kernel has reported a failed bounded wait."""
        if self.dead:
            return False
        if self.dev.type == "cuda" and self.native:
            code = _lib.peek_device_error()
            if code:
                return False
        return True

    def generate(self, reqs: list[GenRequest], stop_when=None, callbacks=None) -> list[GenResult]:
        """Continuous batching with the decode loop on the device: requests are admitted whenever
        a slot and enough KV pages are free (prefilled as a packed batch; their slots join the
        running batch), the batch runs `steps_per_sync` decode steps per host visit (finished
        sequences freeze on the device), and finished sequences leave at the next visit.
        Requests that other threads `submit()` while the call runs join it the same way.

        stop_when(results): checked at every host visit with the finished results so far (rid ->
        GenResult); when it returns True the call aborts the rest (partial rollout: unfinished
        sequences return their tokens so far with finish_reason "abort").
        callbacks: {rid: fn(GenResult)} for requests whose result is delivered by callback (as
        it finishes) instead of in the returned list."""
        if self.dead:
            raise RuntimeError("rollout engine is marked dead (recover it first)")
        from miles_b200.utils import dumper

        if self.speculative is not None:
            with dumper.phase("inference"):
                return self.speculative.generate(reqs, stop_when, callbacks)
        with dumper.phase("inference"):
            return self._generate(reqs, stop_when, callbacks)

    def _generate(self, reqs, stop_when, callbacks) -> list[GenResult]:
        self.resume_memory()
        ds = self.ds
        self.aborted = False
        results: dict[int, GenResult] = {}
        cbs = dict(callbacks or {})
        pending = list(reqs)
        live: dict[int, _Seq] = {}           # slot -> sequence
        free_slots = list(range(self.max_batch - 1, -1, -1))
        t0 = time.perf_counter()
        n_decode_steps = n_prefills = n_syncs = 0
        cur_rows: tuple | None = None
        cur_key = None
        carry: dict[int, tuple] = {}  # rid -> (tokens, logprobs, routed experts) before preemption
        n_preempt = 0

        def finish(res: GenResult):
            if res.rid in carry:
                toks, lps, ex = carry.pop(res.rid)
                res = dataclasses.replace(res, tokens=toks + res.tokens, logprobs=lps + res.logprobs,
                                          routed_experts=res.routed_experts if res.routed_experts is not None
                                          else ex)
            cb = cbs.pop(res.rid, None)
            if cb is not None:
                cb(res)
            else:
                results[res.rid] = res

        with self._lock:
            self._serving = True
        while True:
            with self._lock:
                for r, cb in self._inbox:
                    pending.append(r)
                    cbs[r.rid] = cb
                self._inbox = []
                if self.aborted or not (pending or live):
                    self._serving = False
                    break
            if self.n_moe and any(r.return_routed_experts for r in pending) and ds.out_exp is None:
                if self.cfg.num_experts > 256:
                    raise ValueError("routed-expert recording stores expert ids as uint8 (<= 256 experts)")
                ds.ensure_exp()
            if pending and free_slots:
                new, pending = self._admit(pending, len(free_slots), len(live))
                if new:
                    for sq in new:
                        sq.slot = free_slots.pop()
                        live[sq.slot] = sq
                    imported = [sq for sq in new if sq.handoff is not None]
                    if imported:  # prefilled elsewhere: copy in the K/V rows and the state
                        self._import(imported)
                    new = [sq for sq in new if sq.handoff is None]
                    # packed prefill in chunks of at most `prefill_tokens` tokens (a longer
                    # prompt goes alone): bounds the activation memory next to the KV cache
                    chunk, ntok = [], 0
                    for sq in new:
                        L = len(sq.req.prompt)
                        if chunk and ntok + L > self.prefill_tokens:
                            self._prefill(chunk)
                            n_prefills += 1
                            chunk, ntok = [], 0
                        chunk.append(sq)
                        ntok += L
                    if chunk:
                        self._prefill(chunk)
                        n_prefills += 1
                elif not live:
                    raise RuntimeError("KV cache too small for a single request")
            slots = sorted(live)
            self._filt = self._filter_mode(live.values())
            Bb = self._bucket(len(slots))
            g, st = self._get_steps(Bb)
            rows = tuple(slots) + (self.max_batch,) * (Bb - len(slots))
            key = (Bb, ds.out_exp is not None) + self._filt
            if rows != cur_rows or key != cur_key:
                st["rows"].copy_(torch.tensor(rows, dtype=torch.int32), non_blocking=False)
                cur_rows, cur_key = rows, key
            if self.dev.type == "cuda":
                torch.cuda.nvtx.range_push("decode_steps")
            if g is not None:
                g.replay()
                _lib.add_launches(self.graph_launches[cur_key])
            else:
                for _ in range(self.steps_per_sync):
                    self._step_fn(st)
            if self.dev.type == "cuda":
                torch.cuda.nvtx.range_pop()
            n_decode_steps += self.steps_per_sync
            n_syncs += 1
            done, nout = self._read_flags()
            for sl in slots:
                if done[sl]:
                    sq = live.pop(sl)
                    sq.done = True
                    finish(self._result(sq, int(nout[sl])))
                    self.free_pages.extend(sq.pages)
                    free_slots.append(sl)
            if stop_when is not None and stop_when(results):
                self.aborted = True
            elif self.lazy_pages and live:
                n_preempt += self._grow(live, nout, pending, carry, free_slots)
        if self.aborted:
            done, nout = self._read_flags()
            for sl, sq in list(live.items()):
                finish(self._result(sq, int(nout[sl]), reason="abort"))
                self.free_pages.extend(sq.pages)
                ds.s_done[sl] = 1
            for r in pending:
                finish(GenResult(r.rid, [], [], "abort", None, self.model.weight_version))
        self.stats = {"wall_s": time.perf_counter() - t0, "decode_steps": n_decode_steps,
                      "prefills": n_prefills, "host_syncs": n_syncs, "preemptions": n_preempt}
        return [results[r.rid] for r in reqs if r.rid in results]

    @staticmethod
    def _filter_mode(seqs) -> tuple:
        """(k_max, top_p on) of the sampler for these sequences: k_max is the largest top_k
        rounded up to a power of two (few graph variants), 0 when no row restricts."""
        k = max((s.req.top_k for s in seqs), default=0)
        use_p = any(s.req.top_p < 1.0 for s in seqs)
        kmax = 1 << (int(k) - 1).bit_length() if k > 0 else 0
        return (kmax, use_p)

    def _read_flags(self):
        """Done flags and generated counts of every slot (one small device->host copy)."""
        ds = self.ds
        hf = ds.host_flags
        hf[0].copy_(ds.s_done, non_blocking=True)
        hf[1].copy_(ds.s_nout, non_blocking=True)
        if self.dev.type == "cuda":
            torch.cuda.current_stream(self.dev).synchronize()
        return hf[0].numpy(), hf[1].numpy()

    def _cover(self, plen: int, nout: int, max_new: int) -> int:
        """Pages a sequence must hold before the next graph replay (lazy pages): its fed
        positions plus the replay's steps, capped at its full length."""
        return math.ceil(min(plen + nout + self.steps_per_sync + 1, plen + max_new) / PAGE)

    def _grow(self, live: dict, nout, pending: list, carry: dict, free_slots: list) -> int:
        """Give every live sequence the pages its next `steps_per_sync` decode steps write
        (oldest first); when the pool is empty, preempt the latest admitted sequence: its
        tokens, log-probs and routing so far are kept and it is queued first, to resume by
        re-prefilling prompt + tokens (sampling is keyed by position, so the continuation is the
        same). Returns the number of preemptions."""
        ds = self.ds
        n_pre = 0
        upd_s, upd_i, upd_p = [], [], []
        for sq in sorted(live.values(), key=lambda q: q.order):
            if sq.slot not in live or live[sq.slot] is not sq:
                continue
            want = self._cover(len(sq.req.prompt), int(nout[sq.slot]), sq.req.max_new_tokens)
            while len(sq.pages) < want:
                if self.free_pages:
                    pg = self.free_pages.pop()
                    upd_s.append(sq.slot)
                    upd_i.append(len(sq.pages))
                    upd_p.append(pg)
                    sq.pages.append(pg)
                    continue
                victim = max(live.values(), key=lambda q: q.order)
                n = int(nout[victim.slot])
                res = self._result(victim, n, reason="abort")
                prev = carry.get(victim.req.rid, ([], [], None))
                carry[victim.req.rid] = (prev[0] + res.tokens, prev[1] + res.logprobs,
                                         res.routed_experts if res.routed_experts is not None else prev[2])
                ds.s_done[victim.slot] = 1
                live.pop(victim.slot)
                free_slots.append(victim.slot)
                self.free_pages.extend(victim.pages)
                victim.pages = []
                pending.insert(0, dataclasses.replace(
                    victim.req, prompt=list(victim.req.prompt) + res.tokens,
                    max_new_tokens=victim.req.max_new_tokens - n))
                n_pre += 1
                if victim is sq:
                    break
        if upd_s:
            keep = [j for j, sl in enumerate(upd_s) if sl in live]
            if keep:
                ds.s_pt[torch.tensor([upd_s[j] for j in keep], dtype=torch.long, device=self.dev),
                        torch.tensor([upd_i[j] for j in keep], dtype=torch.long, device=self.dev)] = \
                    torch.tensor([upd_p[j] for j in keep], dtype=torch.int32, device=self.dev)
        return n_pre

    def _admit(self, pending, room: int, n_live: int = 0):
        """Take requests in order while batch slots (`room`) and KV pages last. With lazy pages
        a page per running sequence stays in reserve for growth, so that admitting does not
        immediately force a preemption."""
        wave, rest = [], []
        for r in pending:
            need = math.ceil((len(r.prompt) + r.max_new_tokens) / PAGE)
            if need > self.max_pages_per_seq:
                raise ValueError(f"request needs {need} pages > max_pages_per_seq")
            reserve = 0
            if self.lazy_pages:
                need = self._cover(len(r.prompt), 1, r.max_new_tokens)
                reserve = n_live + len(wave) if (n_live or wave) else 0
            if not rest and len(wave) < room and need + reserve <= len(self.free_pages):
                sq = _Seq(getattr(r, "req", r), [self.free_pages.pop() for _ in range(need)])
                if isinstance(r, PrefillHandoff):
                    sq.handoff = r
                wave.append(sq)
            else:
                rest.append(r)  # keep arrival order: no request overtakes an earlier one
        return wave, rest

    def _slot(self, s: _Seq, pos: int) -> int:
        return s.pages[pos // PAGE] * PAGE + pos % PAGE

    def _prefill(self, wave: list[_Seq]) -> None:
        """Packed prefill of newly admitted sequences; samples their first token and writes
        their slots' device state (nothing is read back)."""
        dev, ds = self.dev, self.ds
        cu = [0]
        toks, slots = [], []
        for s in wave:
            toks.extend(s.req.prompt)
            slots.extend(self._slot(s, p) for p in range(len(s.req.prompt)))
            cu.append(len(toks))
        meta = VarlenMeta(cu, dev)
        rec = [] if (self.n_moe and ds.out_exp is not None) else None
        nvtx = dev.type == "cuda"
        if nvtx:
            torch.cuda.nvtx.range_push("prefill")
        sl = torch.tensor([s.slot for s in wave], dtype=torch.int64, device=dev)
        h = self.model.forward_prefill(torch.tensor(toks, dtype=torch.int32, device=dev), meta,
                                       self.cache, torch.tensor(slots, dtype=torch.int64, device=dev),
                                       record=rec, state_rows=sl)
        last = torch.tensor([c - 1 for c in cu[1:]], dtype=torch.long, device=dev)
        invt_h = [1.0 / s.req.temperature if s.req.temperature > 0 else 0.0 for s in wave]
        seed_h = [s.req.seed for s in wave]
        plen_h = [len(s.req.prompt) for s in wave]
        inv_t = torch.tensor(invt_h, dtype=torch.float32, device=dev)
        seeds = torch.tensor(seed_h, dtype=torch.int64, device=dev)
        posn = torch.tensor(plen_h, dtype=torch.int32, device=dev)
        kmax, use_p = self._filter_mode(wave)
        topk = torch.tensor([s.req.top_k for s in wave], dtype=torch.int32, device=dev)
        topp = torch.tensor([float(s.req.top_p) for s in wave], dtype=torch.float32, device=dev)
        tok, lp = sample_from_hidden(h.index_select(0, last).contiguous(), self.model.lm_head_weight(),
                                     inv_t, seeds, posn, top_k=topk if kmax else None,
                                     top_p=topp if use_p else None, k_max=kmax)
        self._set_slots(wave, tok, lp, inv_t, seeds, posn, topk, topp)
        if rec:
            ex = torch.stack(rec, 1).to(torch.uint8)  # [T, L_moe, k]
            for b, s in enumerate(wave):
                if s.req.return_routed_experts:
                    ds.out_exp[s.slot, :plen_h[b]] = ex[cu[b]:cu[b + 1]]
        if nvtx:
            torch.cuda.nvtx.range_pop()

    def _sampling_params(self, wave: list[_Seq]):
        dev = self.dev
        inv_t = torch.tensor([1.0 / s.req.temperature if s.req.temperature > 0 else 0.0 for s in wave],
                             dtype=torch.float32, device=dev)
        seeds = torch.tensor([s.req.seed for s in wave], dtype=torch.int64, device=dev)
        posn = torch.tensor([len(s.req.prompt) for s in wave], dtype=torch.int32, device=dev)
        topk = torch.tensor([s.req.top_k for s in wave], dtype=torch.int32, device=dev)
        topp = torch.tensor([float(s.req.top_p) for s in wave], dtype=torch.float32, device=dev)
        return inv_t, seeds, posn, topk, topp

    def _check_pd(self) -> None:
        c = self.cfg
        if c.kv_lora_rank or c.linear_attn_interval:
            raise ValueError("prefill / decode hand-off supports standard K/V caches only "
                             "(not MLA latents or Gated DeltaNet states)")

    def _import(self, wave: list[_Seq]) -> None:
        """Admit sequences prefilled by another engine: their prompt K/V rows are written into
        this engine's pages and their slots get the state `_prefill` would have set."""
        self._check_pd()
        dev, ds, cache = self.dev, self.ds, self.cache
        for s in wave:
            h = s.handoff
            P = len(s.req.prompt)
            rows = torch.tensor([self._slot(s, p) for p in range(P)], dtype=torch.int64, device=dev)
            j = 0
            for i in range(self.cfg.num_layers):
                cache.k[i].index_copy_(0, rows, h.k[j].to(dev, cache.k[i].dtype))
                cache.v[i].index_copy_(0, rows, h.v[j].to(dev, cache.v[i].dtype))
                j += 1
            if h.experts is not None and s.req.return_routed_experts and ds.out_exp is not None:
                ds.out_exp[s.slot, :P] = torch.from_numpy(np.asarray(h.experts)).to(dev, torch.uint8)
        tok = torch.tensor([s.handoff.token for s in wave], dtype=torch.int32, device=dev)
        lp = torch.tensor([s.handoff.logprob for s in wave], dtype=torch.float32, device=dev)
        self._set_slots(wave, tok, lp, *self._sampling_params(wave))

    def prefill_handoffs(self, reqs: list[GenRequest]) -> list[PrefillHandoff]:
        """Prefill role of prefill / decode disaggregation: prefill every request (packed, as
        many at a time as slots and pages allow), sample its first token and return the
        hand-offs; this engine keeps nothing. A decode engine continues them with
        `generate(handoffs)` (the same tokens a single engine would produce)."""
        self._check_pd()
        self.resume_memory()
        ds = self.ds
        if self.n_moe and any(r.return_routed_experts for r in reqs):
            ds.ensure_exp()
        out: dict[int, PrefillHandoff] = {}
        pending = list(reqs)
        while pending:
            new, pending = self._admit(pending, self.max_batch)
            if not new:
                raise RuntimeError("KV cache too small for a single request")
            for j, sq in enumerate(new):
                sq.slot = j
            chunk, ntok = [], 0
            for sq in new:
                if chunk and ntok + len(sq.req.prompt) > self.prefill_tokens:
                    self._prefill(chunk)
                    chunk, ntok = [], 0
                chunk.append(sq)
                ntok += len(sq.req.prompt)
            self._prefill(chunk)
            for sq in new:
                P = len(sq.req.prompt)
                rows = torch.tensor([self._slot(sq, p) for p in range(P)], dtype=torch.int64,
                                    device=self.dev)
                k = [self.cache.k[i].index_select(0, rows) for i in range(self.cfg.num_layers)]
                v = [self.cache.v[i].index_select(0, rows) for i in range(self.cfg.num_layers)]
                ex = None
                if sq.req.return_routed_experts and ds.out_exp is not None:
                    ex = ds.out_exp[sq.slot, :P].clone().cpu().numpy()  # the slot is reused
                out[sq.req.rid] = PrefillHandoff(sq.req, k, v, int(ds.s_tok[sq.slot]),
                                                 float(ds.out_lp[sq.slot, 0].detach()), ex)
                ds.s_done[sq.slot] = 1
                self.free_pages.extend(sq.pages)
        return [out[r.rid] for r in reqs]

    def _set_slots(self, wave: list[_Seq], tok, lp, inv_t, seeds, posn, topk, topp) -> None:
        """Device state of freshly prefilled (or imported) sequences: page-table rows, sampling
        parameters, the first sampled token and its log-prob, done flags."""
        dev, ds = self.dev, self.ds
        sl = torch.tensor([s.slot for s in wave], dtype=torch.int64, device=dev)
        n = len(wave)
        pt = np.zeros((n, self.max_pages_per_seq), np.int32)
        stop = np.full((n, _NSTOP), -1, np.int32)
        for b, s in enumerate(wave):
            pt[b, :len(s.pages)] = s.pages
            ids = list(s.req.stop_token_ids)
            if len(ids) > _NSTOP:
                raise ValueError(f"at most {_NSTOP} stop token ids per request")
            stop[b, :len(ids)] = ids
        maxnew = torch.tensor([s.req.max_new_tokens for s in wave], dtype=torch.int32, device=dev)
        stop_d = torch.from_numpy(stop).to(dev)
        ds.s_pt[sl] = torch.from_numpy(pt).to(dev)
        ds.s_stop[sl] = stop_d
        ds.s_invt[sl] = inv_t
        ds.s_seed[sl] = seeds
        ds.s_topk[sl] = topk
        ds.s_topp[sl] = topp
        ds.s_maxnew[sl] = maxnew
        ds.s_rec[sl] = torch.tensor([int(s.req.return_routed_experts) for s in wave],
                                    dtype=torch.int32, device=dev)
        ds.s_tok[sl] = tok
        ds.s_pos[sl] = posn
        ds.s_nout[sl] = 1
        ds.out_tok[sl, 0] = tok
        ds.out_lp[sl, 0] = lp
        first_done = (maxnew <= 1) | (stop_d == tok[:, None]).any(1)
        ds.s_done[sl] = first_done.int()

    def _result(self, s: _Seq, n: int, reason: str | None = None) -> GenResult:
        ds = self.ds
        n = max(0, min(n, ds.max_len))
        toks = ds.out_tok[s.slot, :n].tolist()
        lps = ds.out_lp[s.slot, :n].tolist()
        if reason is None:
            reason = "stop" if (toks and toks[-1] in s.req.stop_token_ids) else "length"
        ex = None
        if s.req.return_routed_experts and ds.out_exp is not None and n > 0:
            rows = len(s.req.prompt) + n - 1
            ex = ds.out_exp[s.slot, :rows].to(torch.int32).cpu().numpy()
        return GenResult(s.req.rid, toks, lps, reason, ex, self.model.weight_version)
