"""Training actor: packing, log-prob collection, advantage estimation and the policy update.

One `Actor` per GPU process. Samples arrive with their prompt/response tokens, loss mask,
reward-derived advantage and the rollout log-probs the engine recorded. A training step:

  1. pack samples into micro-batches of at most `max_tokens_per_gpu` tokens (first-fit
     decreasing, thd layout: no padding inside a micro-batch),
  2. old log-probs: a no-grad forward (or the rollout log-probs with --use-rollout-logprobs);
     with colocated weights they are bitwise equal to the engine's, which is checked,
  3. per micro-batch: recompute-checkpointed forward (+ R3 routing replay), chunked LM-head
     log-prob/entropy, fused clipped policy loss, backward into the flat gradient buffer,
  4. data-parallel gradient reduction (when the world is larger than one) and the flat Adam.

Reference: megatron_utils/actor.py (train_actor :367-466), training_utils/data.py
(get_batch / DataIterator :86-418), training_utils/loss.py (policy_loss_function :500-716,
loss scaling :828-927), megatron_utils/model.py (train_one_step :318-490).
"""
from __future__ import annotations

import dataclasses
import math
import time
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.distributed as dist

from miles_b200.models.transformer import Transformer
from miles_b200.ops.gemm import clear_main_grads, register_main_grad
from miles_b200.parallel.tp import tp_partial_param_names, tp_replicated_ranges
from miles_b200.ops.attention import VarlenMeta, to_device
from miles_b200.ops.rl import METRIC_NAMES, PolicyLossCfg, policy_loss
from miles_b200.trainer.lr_scheduler import LRSchedule
from miles_b200.trainer.optimizer import FlatAdam
from miles_b200.utils.misc import load_function


@dataclass
class TrainItem:
    tokens: list[int]
    prompt_len: int
    advantage: float | list[float] = 0.0
    loss_mask: list[int] | None = None          # over the response tokens
    rollout_logp: list[float] | None = None
    old_logp: list[float] | None = None
    ref_logp: list[float] | None = None
    routed_experts: np.ndarray | None = None    # [len(tokens)-1, L_moe, k] int32
    # response index from which rollout_logp was produced by the current weights (partial
    # rollout resumes a sample under newer weights; earlier tokens are off-policy)
    fresh_from: int = 0

    @property
    def resp_len(self) -> int:
        return len(self.tokens) - self.prompt_len


@dataclass
class ActorConfig:
    lr: float = 1e-6
    betas: tuple = (0.9, 0.98)
    weight_decay: float = 0.0
    clip_grad: float = 1.0
    max_tokens_per_gpu: int = 16384
    loss: PolicyLossCfg = field(default_factory=PolicyLossCfg)
    entropy_coef: float = 0.0
    per_token_loss: bool = False
    mtp_loss_scale: float = 0.0      # weight of the multi-token prediction loss (model.mtp_train)
    temperature: float = 1.0
    use_rollout_logprobs: bool = False
    # old log-probs from the training forward itself (one optimizer step per rollout): the
    # separate no-grad pass would recompute the same values bit for bit (batch-invariant
    # kernels, unchanged weights), so the training forward's detached log-probs are used
    old_logp_from_forward: bool = False
    use_routing_replay: bool = False
    grad_dtype: torch.dtype = torch.bfloat16
    optimizer_placement: str = "auto"
    logprob_chunk: int = 4096
    adam_eps: float = 1e-8
    # micro-batching: "ffd" (first-fit decreasing under max_tokens_per_gpu), "balanced"
    # (--use-dynamic-batch-size: fewest micro-batches under the budget, Karmarkar-Karp balanced
    # token totals) or "fixed" (--micro-batch-size samples per micro-batch, in order)
    micro_batching: str = "ffd"
    micro_batch_size: int = 1
    log_probs_max_tokens_per_gpu: int | None = None
    lr_schedule: "LRSchedule | None" = None   # None: constant `lr`
    tis_args: object = None   # namespace handed to a custom TIS function (e.g. MIS settings)
    memory_margin_bytes: int = 0   # device memory kept free when placing the optimizer state
    # colocated: park device-placed optimizer state in pinned host memory while rolling out
    # (released with the gradients, back before the optimizer step)
    offload_optimizer: bool = False
    # DP gradient reduce-scatter: "nccl", or "peer" (fused kernel over a resident symmetric
    # gradient buffer; sharded bf16 gradients on CUDA)
    grad_reduce: str = "nccl"


def pack_microbatches(lengths: list[int], max_tokens: int) -> list[list[int]]:
    """First-fit-decreasing bin packing of sample indices under a token budget."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    bins: list[list[int]] = []
    loads: list[int] = []
    for i in order:
        L = lengths[i]
        for b in range(len(bins)):
            if loads[b] + L <= max_tokens:
                bins[b].append(i)
                loads[b] += L
                break
        else:
            bins.append([i])
            loads.append(L)
    return [sorted(b) for b in bins]


def make_micro_batches(lengths: list[int], cfg: "ActorConfig", budget: int | None = None) -> list[list[int]]:
    """Micro-batches (lists of sample indices) under the configured policy."""
    budget = budget or cfg.max_tokens_per_gpu
    if cfg.micro_batching == "balanced":
        from miles_b200.utils.seqlen_balancing import balanced_micro_batches

        return balanced_micro_batches(lengths, budget)
    if cfg.micro_batching == "fixed":
        m = max(1, cfg.micro_batch_size)
        return [list(range(i, min(i + m, len(lengths)))) for i in range(0, len(lengths), m)]
    return pack_microbatches(lengths, budget)


def _seg_mean(x: torch.Tensor, mask: torch.Tensor, seg: torch.Tensor, nseq: int) -> torch.Tensor:
    """Per-token broadcast of the masked mean of x over each token's sequence (differentiable)."""
    num = torch.zeros(nseq, dtype=x.dtype, device=x.device).index_add(0, seg, x)
    den = torch.zeros(nseq, dtype=x.dtype, device=x.device).index_add(0, seg, mask).clamp_min(1.0)
    return (num / den).index_select(0, seg)


class Actor:
    def __init__(self, model: Transformer, cfg: ActorConfig, dp_group=None):
        self.model = model
        self.cfg = cfg
        self.dp_group = dp_group
        self.dev = model.device
        self.grad_flat: torch.Tensor | None = None
        self.opt: FlatAdam | None = None
        self.timers: dict[str, float] = {}
        self._custom_loss = None
        self._custom_tis = None
        self._pg_reducer = None
        self._peer_grads = None
        self._host_state = self._prefetch_host_state()

    # ------------------------------------------------------------------ memory
    def _ensure_grads(self):
        if self.model.lora is not None:
            # LoRA: base weights frozen, only the adapters train (no flat gradient buffer)
            if self.opt is None:
                from miles_b200.models.lora import LoRAOptimizer

                for p in self.model.params.values():
                    p.requires_grad_(False)
                self.opt = LoRAOptimizer(self.model.lora, self.cfg.lr, self.cfg.betas,
                                         self.cfg.weight_decay, self.cfg.clip_grad, self.dp_group)
            return
        if self.grad_flat is None:
            n = self.model.flat.numel()
            if self._use_peer_grads():
                if self._peer_grads is None:
                    from miles_b200.parallel.symm import PeerGradBuffer

                    self._peer_grads = PeerGradBuffer(n, self.dp_group, self.dev)
                self.grad_flat = self._peer_grads.tensor
                self.grad_flat.zero_()
            else:
                self.grad_flat = torch.zeros(n, dtype=self.cfg.grad_dtype, device=self.dev)
            for s in self.model.specs:
                g = self.grad_flat[s.offset:s.offset + s.numel].view(s.shape)
                self.model.params[s.name].main_grad = g
                register_main_grad(self.model.params[s.name], g)
        if self.opt is not None:
            self.opt.g = self.grad_flat
        else:
            self.opt = FlatAdam(self.model.flat, self.grad_flat, lr=self.cfg.lr,
                                betas=self.cfg.betas, eps=self.cfg.adam_eps,
                                weight_decay=self.cfg.weight_decay,
                                clip_grad=self.cfg.clip_grad, placement=self.cfg.optimizer_placement,
                                host_state=self._host_state,
                                memory_margin=self.cfg.memory_margin_bytes,
                                dp_group=self.dp_group if self._sharded() else None,
                                peer_grads=self._peer_grads,
                                **self._norm_scope())

    def _prefetch_host_state(self):
        """Start page-locking the host-resident Adam state now (under the first rollout) when
        the optimizer will keep it on the host: FlatAdam's 'auto' rule with the gradient
        buffer that _ensure_grads allocates first."""
        m, cfg = self.model, self.cfg
        if m.device.type != "cuda" or m.lora is not None or cfg.optimizer_placement == "device":
            return None
        n = m.flat.numel()
        world = dist.get_world_size(self.dp_group) if self._sharded() else 1
        ns = n // world
        if cfg.optimizer_placement == "auto":
            free, _ = torch.cuda.mem_get_info(m.device)
            free -= cfg.memory_margin_bytes
            grad_bytes = n * torch.empty((), dtype=cfg.grad_dtype).element_size()
            if not 12 * ns > 0.8 * (free - grad_bytes):
                return None
        from miles_b200.utils.host_memory import BackgroundPinned

        return (BackgroundPinned(ns, torch.bfloat16), BackgroundPinned(ns, torch.bfloat16))

    def _norm_scope(self) -> dict:
        """Gradient-norm group of model-parallel ranks and the flat ranges this rank leaves out;
        under expert parallelism the experts' part is summed over the groups that split them."""
        m = self.model
        out = {}
        if m.ep is not None:
            groups = ([m.tp.group] if m.tp is not None and m.expert_tp > 1 else []) + [m.ep.group]
            out["expert_norm"] = (m.dense_numel, groups)
        if m.tp is not None:
            out.update({"norm_group": m.tp.group,
                        "norm_exclude": tp_replicated_ranges(m) if m.tp.rank != 0 else []})
            return out
        if m.ep is not None:
            return out
        if m.pp is not None:
            ex = []
            if m.cfg.tie_embeddings and m.pp.is_last and not m.pp.is_first:
                sp = next(s for s in m.specs if s.name == "embed_tokens.weight")
                ex.append((sp.offset, sp.offset + sp.numel))
            return {"norm_group": m.pp.group, "norm_exclude": ex}
        return {}

    def _use_peer_grads(self) -> bool:
        return (self.cfg.grad_reduce == "peer" and self._sharded() and self.dev.type == "cuda"
                and self.cfg.grad_dtype == torch.bfloat16)

    def _sharded(self) -> bool:
        """Optimizer sharded over the data-parallel group (ZeRO-1): every rank holds the whole
        flat buffer (no expert parallelism) and there is more than one rank."""
        return (self.dp_group is not None and dist.get_world_size(self.dp_group) > 1
                and self.model.ep is None and self.model.lora is None)

    def release_grads(self):
        """Free the gradient buffer (colocated mode: give the memory to the KV cache)."""
        for s in self.model.specs:
            p = self.model.params[s.name]
            if hasattr(p, "main_grad"):
                del p.main_grad
        clear_main_grads()
        self.grad_flat = None
        if self.opt is not None:
            self.opt.g = None
            if self.cfg.offload_optimizer and hasattr(self.opt, "offload"):
                self.opt.offload()
        if self.dev.type == "cuda":
            torch.cuda.empty_cache()

    # ------------------------------------------------------------------ batching
    def _mb_inputs(self, items: list[TrainItem]):
        toks = [np.asarray(it.tokens, dtype=np.int32) for it in items]
        lens = np.array([len(t) for t in toks], dtype=np.int64)
        cu = np.concatenate([[0], np.cumsum(lens)])
        # hidden at position p predicts token p+1: response tokens P..L-1 <- rows P-1..L-2
        sel = np.concatenate([np.arange(cu[i] + it.prompt_len - 1, cu[i + 1] - 1, dtype=np.int64)
                              for i, it in enumerate(items)]) if items else np.zeros(0, np.int64)
        tgt = np.concatenate([t[it.prompt_len:] for t, it in zip(toks, items)]) if items else \
            np.zeros(0, np.int32)
        dev = self.dev
        meta = VarlenMeta(cu.tolist(), dev)
        return (to_device(np.concatenate(toks) if toks else np.zeros(0, np.int32), dev), meta,
                to_device(sel, dev), to_device(tgt.astype(np.int32), dev))

    def _replay(self, items: list[TrainItem]):
        if not self.cfg.use_routing_replay or not items or items[0].routed_experts is None:
            return None
        parts = []
        for it in items:
            ex = it.routed_experts
            # the last token never went through the model during rollout; repeat its predecessor
            ex = np.concatenate([ex, ex[-1:]], 0)[: len(it.tokens)]
            parts.append(ex)
        return to_device(np.concatenate(parts, 0), self.dev)

    # ------------------------------------------------------------------ log-probs
    @torch.no_grad()
    def compute_logprobs(self, items: list[TrainItem]) -> list[np.ndarray]:
        """Forward-only response log-probs of every item (old / ref log-probs)."""
        from miles_b200.utils import dumper

        with dumper.phase("fwd_only"):
            return self._compute_logprobs(items)

    def _compute_logprobs(self, items: list[TrainItem]) -> list[np.ndarray]:
        out: list[np.ndarray | None] = [None] * len(items)
        if self.model.pp is not None:
            return self._logprobs_pp(items)
        pending = []
        for mb in make_micro_batches([len(it.tokens) for it in items], self.cfg,
                                     self.cfg.log_probs_max_tokens_per_gpu):
            sub = [items[i] for i in mb]
            tok, meta, sel, tgt = self._mb_inputs(sub)
            lp, _ = self.model.selected_logprob(tok, meta, sel, tgt, self.cfg.temperature,
                                                self.cfg.logprob_chunk, self._replay(sub))
            pending.append((mb, lp.float()))
        # one device -> host copy at the end (a copy per micro-batch would stall the host on
        # every one while the next micro-batch's inputs could already be queued)
        if pending:
            flat = torch.cat([lp for _, lp in pending]).cpu().numpy()
            o = 0
            for mb, _ in pending:
                for i in mb:
                    n = items[i].resp_len
                    out[i] = flat[o:o + n]
                    o += n
        return out

    @torch.no_grad()
    def _logprobs_pp(self, items):
        from miles_b200.ops.logprob import lm_head_logprob
        from miles_b200.parallel.pp import run_forward_only, run_interleaved

        model, cfg = self.model, self.cfg
        mbs = make_micro_batches([len(it.tokens) for it in items], cfg, cfg.log_probs_max_tokens_per_gpu)
        subs = [[items[i] for i in mb] for mb in mbs]
        ins = [self._mb_inputs(sub) for sub in subs]
        shapes = [(x[0].shape[0], model.cfg.hidden_size) for x in ins]
        out: list = [None] * len(items)

        V = model.pp.vpp

        def forward(j, h, c=None):
            tok, meta, sel, tgt = ins[j]
            y = model.forward_train(tok, meta, replay_experts=self._replay(subs[j]), hidden_in=h,
                                    chunk=c)
            if model.is_last and (c is None or c == V - 1):
                lp, _ = lm_head_logprob(y.index_select(0, sel), model.lm_head_weight(), tgt,
                                        cfg.temperature, cfg.logprob_chunk)
                lp = lp.float().cpu().numpy()
                o = 0
                for i in mbs[j]:
                    n = items[i].resp_len
                    out[i] = lp[o:o + n]
                    o += n
            return y

        if V > 1:
            run_interleaved(model.pp, len(ins), shapes, model.dtype, self.dev,
                            lambda j, c, h: forward(j, h, c), None)
        else:
            run_forward_only(model.pp, len(ins), shapes, model.dtype, self.dev, forward)
        box = [out]
        dist.broadcast_object_list(box, model.pp.ranks[-1], group=model.pp.group)
        return box[0]

    # ------------------------------------------------------------------ train
    def train_step(self, items: list[TrainItem], global_num_samples: int | None = None,
                   global_num_tokens: int | None = None) -> dict:
        from miles_b200.utils import dumper

        with dumper.phase("fwd_bwd"):
            return self._train_step(items, global_num_samples, global_num_tokens)

    def _train_step(self, items: list[TrainItem], global_num_samples: int | None = None,
                    global_num_tokens: int | None = None) -> dict:
        cfg = self.cfg
        self._ensure_grads()
        model = self.model
        t0 = time.perf_counter()
        if self.grad_flat is not None:
            self.grad_flat.zero_()
        n_samples = global_num_samples or len(items)
        n_tokens = global_num_tokens or sum(
            (sum(it.loss_mask) if it.loss_mask is not None else it.resp_len) for it in items)
        metrics = torch.zeros(len(METRIC_NAMES) + 1, dtype=torch.float64, device=self.dev)
        # sum |old - rollout|, count; the same over tokens sampled under the current weights
        self._parity = torch.zeros(4, dtype=torch.float64, device=self.dev)
        mbs = make_micro_batches([len(it.tokens) for it in items], cfg)
        mtp_total = torch.zeros((), dtype=torch.float32, device=self.dev)
        if model.pp is not None:
            self._train_pp(items, mbs, n_samples, n_tokens, metrics)
        for mb in ([] if model.pp is not None else mbs):
            sub = [items[i] for i in mb]
            prep = self._mb_prepare(sub, n_samples, n_tokens)
            lp, ent = model.selected_logprob(prep["tok"], prep["meta"], prep["sel"], prep["tgt"],
                                             cfg.temperature, cfg.logprob_chunk, self._replay(sub))
            loss = self._mb_loss(prep, lp, ent, metrics)
            if model.mtp_train and cfg.mtp_loss_scale:
                lm = model.mtp_loss(prep["tok"], prep["meta"], prep["sel"], prep["tgt"], prep["wgt"],
                                    cfg.temperature, cfg.logprob_chunk)
                loss = loss + cfg.mtp_loss_scale * lm
                mtp_total += lm.detach().float()
            loss.backward()
        model._mtp_h = None  # the last microbatch's final hidden is not kept past the step
        # parameters whose gradient came through autograd (embedding, norms) -> flat buffer
        for name, p in model.params.items():
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(p.main_grad.dtype))
                p.grad = None
        t1 = time.perf_counter()
        if model.tp is not None:
            for name in tp_partial_param_names(model):
                dist.all_reduce(model.params[name].main_grad, group=model.tp.group)
        if (self.dp_group is not None and dist.get_world_size(self.dp_group) > 1
                and not self._sharded() and model.lora is None):
            self._reduce_grads()
        if cfg.lr_schedule is not None:
            # the LR of this step from the samples consumed before it (Megatron order)
            self.opt.lr = cfg.lr_schedule.lr()
            cfg.lr_schedule.advance(n_samples)
        self.opt.step()  # sharded: reduce-scatter + shard update + all-gather inside
        model.weight_version += 1
        out = {k: float(v) for k, v in zip(METRIC_NAMES + ["entropy"], metrics.tolist())}
        if cfg.old_logp_from_forward:
            s_, n_, sf, nf = self._parity.tolist()
            out["train_rollout_logprob_abs_diff"] = s_ / max(n_, 1.0)
            out["train_rollout_logprob_abs_diff_current_weights"] = sf / max(nf, 1.0)
            out["train_rollout_logprob_current_weight_tokens"] = nf
        out["grad_norm"] = float(self.opt.grad_norm())
        out["lr"] = float(self.opt.lr)
        if model.mtp_train and cfg.mtp_loss_scale:
            out["mtp_loss"] = float(mtp_total)
        out["num_microbatches"] = len(mbs)
        self.timers["train_fwd_bwd"] = t1 - t0
        self.timers["train_total"] = time.perf_counter() - t0
        return out

    # ------------------------------------------------------------------ micro-batch pieces
    def _mb_prepare(self, sub: list[TrainItem], n_samples: int, n_tokens: int) -> dict:
        """Host-built inputs and per-token loss terms of one micro-batch."""
        cfg = self.cfg
        tok, meta, sel, tgt = self._mb_inputs(sub)
        adv, old, roll, ref, wgt, fresh = [], [], [], [], [], []
        for it in sub:
            n = it.resp_len
            fresh.append((np.arange(n) >= it.fresh_from).astype(np.float32))
            mask = np.asarray(it.loss_mask if it.loss_mask is not None else [1] * n, np.float32)
            a = it.advantage
            adv.append(np.full(n, a, np.float32) if np.isscalar(a) else np.asarray(a, np.float32))
            if it.old_logp is not None:
                old.append(np.asarray(it.old_logp, np.float32))
            elif it.rollout_logp is not None:
                old.append(np.asarray(it.rollout_logp, np.float32))
            else:
                old.append(np.zeros(n, np.float32))
            roll.append(np.asarray(it.rollout_logp if it.rollout_logp is not None else old[-1], np.float32))
            if it.ref_logp is not None:
                ref.append(np.asarray(it.ref_logp, np.float32))
            if cfg.per_token_loss:
                wgt.append(mask / max(n_tokens, 1))
            else:
                wgt.append(mask / max(mask.sum(), 1.0) / n_samples)
        T = lambda xs: to_device(np.concatenate(xs), self.dev)  # noqa: E731
        seg = to_device(np.repeat(np.arange(len(sub)), [it.resp_len for it in sub]), self.dev)
        return {"tok": tok, "meta": meta, "sel": sel, "tgt": tgt, "n": len(sub), "seg": seg,
                "old": T(old), "adv": T(adv), "wgt": T(wgt), "fresh": T(fresh),
                "roll": T(roll) if any(r is not None for r in roll) else None,
                "ref": T(ref) if ref and cfg.loss.kl_type != "none" else None}

    def _mb_loss(self, prep: dict, lp, ent, metrics: torch.Tensor):
        cfg = self.cfg
        if cfg.old_logp_from_forward:
            prep = dict(prep, old=lp.detach().float())
            if prep["roll"] is not None:
                mask = (prep["wgt"] > 0).double()
                d = (prep["old"] - prep["roll"]).abs().double()
                self._parity[0] += (d * mask).sum()
                self._parity[1] += mask.sum()
                fm = mask * prep["fresh"].double()
                self._parity[2] += (d * fm).sum()
                self._parity[3] += fm.sum()
        self._cur_total_lens = [b - a for a, b in zip(prep["meta"].cu_list[:-1], prep["meta"].cu_list[1:])]
        loss, m = self._loss(lp, ent, prep["seg"], prep["n"], prep["old"], prep["adv"], prep["wgt"],
                             prep["roll"], prep["ref"])
        if cfg.entropy_coef:
            loss = loss - cfg.entropy_coef * (ent * prep["wgt"]).sum()
        metrics[: len(METRIC_NAMES)] += m.double().to(self.dev)
        metrics[-1] += ((ent.detach() * prep["wgt"]).sum()).double()
        return loss

    def _train_pp(self, items, mbs, n_samples, n_tokens, metrics):
        """One training pass over the micro-batches through the 1F1B pipeline; the loss and the
        metrics live on the last stage, which broadcasts the metrics to the other stages."""
        from miles_b200.ops.logprob import lm_head_logprob
        from miles_b200.parallel.pp import reduce_tied_embedding, run_1f1b, run_interleaved

        model, cfg = self.model, self.cfg
        subs = [[items[i] for i in mb] for mb in mbs]
        preps = [self._mb_prepare(sub, n_samples, n_tokens) for sub in subs]
        shapes = [(p["tok"].shape[0], model.cfg.hidden_size) for p in preps]

        V = model.pp.vpp

        def forward(j, h, c=None):
            p = preps[j]
            out = model.forward_train(p["tok"], p["meta"], replay_experts=self._replay(subs[j]),
                                      hidden_in=h, chunk=c)
            if not (model.is_last and (c is None or c == V - 1)):
                return out
            lp, ent = lm_head_logprob(out.index_select(0, p["sel"]), model.lm_head_weight(), p["tgt"],
                                      cfg.temperature, cfg.logprob_chunk)
            return self._mb_loss(p, lp, ent, metrics)

        def backward(j, out, g):
            if g is None:
                out.backward()
            else:
                out.backward(g)

        if V > 1:
            run_interleaved(model.pp, len(preps), shapes, model.dtype, self.dev,
                            lambda j, c, h: forward(j, h, c), lambda j, c, out, g: backward(j, out, g))
        else:
            run_1f1b(model.pp, len(preps), shapes, model.dtype, self.dev, forward, backward)
        for name, p in model.params.items():  # autograd-held grads -> flat buffer before the tie
            if p.grad is not None:
                p.main_grad.add_(p.grad.to(p.main_grad.dtype))
                p.grad = None
        reduce_tied_embedding(model)
        dist.broadcast(metrics, model.pp.ranks[-1], group=model.pp.group)

    # ------------------------------------------------------------------ losses
    def _loss(self, lp, ent, seg, nseq, old, adv, wgt, roll, ref):
        """Loss of one micro-batch (token-level tensors over its response tokens; `seg` maps a
        token to its sample). Returns (loss, metrics [len(METRIC_NAMES)] weighted sums)."""
        cfg = self.cfg
        lc = cfg.loss
        if lc.loss_type == "sft_loss":
            # SFT: negative log-likelihood of the (loss-masked) response tokens
            loss = -(lp * wgt).sum()
            m = torch.zeros(len(METRIC_NAMES), dtype=torch.float32, device=lp.device)
            m[0] = loss.detach()
            m[len(METRIC_NAMES) - 1] = wgt.sum()
            return loss, m
        if lc.loss_type == "custom_loss":
            if self._custom_loss is None:
                self._custom_loss = load_function(lc.custom_loss_path)
            return self._custom_loss(lp=lp, entropy=ent, old_log_probs=old, advantages=adv,
                                     weights=wgt, rollout_log_probs=roll, ref_log_probs=ref,
                                     segments=seg, cfg=lc)
        w = wgt
        mask = (wgt > 0).float()
        if lc.use_opsm:
            # off-policy sequence masking: drop sequences with negative advantage whose
            # sequence-level KL(old || current) exceeds opsm_delta
            kl = _seg_mean((old - lp.detach()) * mask, mask, seg, nseq)
            w = w * (1.0 - ((adv < 0) & (kl > lc.opsm_delta)).float())
        if lc.use_tis and lc.custom_tis_path and roll is not None:
            if self._custom_tis is None:
                self._custom_tis = load_function(lc.custom_tis_path)
            # reference hook signature: scales pg_loss; applied to the (detached) weights
            sizes = torch.bincount(seg, minlength=nseq).tolist()
            sp = lambda x: list(torch.split(x, sizes))  # noqa: E731  (per-sample tensors)
            scaled, masks, _ = self._custom_tis(cfg.tis_args if cfg.tis_args is not None else lc,
                                                pg_loss=torch.ones_like(lp), train_log_probs=sp(old),
                                                rollout_log_probs=sp(roll), loss_masks=sp(mask))
            w = w * scaled.detach()
            if masks is not None:  # rejection (mask mode / rejection sampling) drops tokens
                w = w * torch.cat([mm.float() for mm in masks]).to(w.device)
            lc = dataclasses.replace(lc, use_tis=False)
        lp_in, old_in = lp, old
        if lc.gspo:
            # GSPO: sequence-level importance ratio exp(mean_t(logp - old)) on every token
            lp_in = _seg_mean(lp * mask, mask, seg, nseq)
            old_in = _seg_mean(old * mask, mask, seg, nseq)
        reducer = None
        if lc.custom_pg_loss_reducer_path:
            # custom reducer: fn(total_lengths, response_lengths, loss_masks, per_token_loss)
            # returns a callable over the concatenated per-token pg loss (reference
            # training_utils/loss.py:644-652)
            if self._pg_reducer is None:
                self._pg_reducer = load_function(lc.custom_pg_loss_reducer_path)
            rl = torch.bincount(seg, minlength=nseq).tolist()
            masks = list(torch.split(mask, rl))
            tl = getattr(self, "_cur_total_lens", None) or rl
            reducer = self._pg_reducer(tl, rl, masks, cfg.per_token_loss)
        return policy_loss(lp_in, old_in, adv, w, lc, roll if lc.use_tis else None, ref, reducer)

    def _reduce_grads(self):
        """Sum gradients over data-parallel ranks (replicated region) and expert-data-parallel
        ranks (expert region, none when EP == world)."""
        dense = self.grad_flat[: self.model.dense_numel]
        dist.all_reduce(dense, group=self.dp_group)
        ep_dp = getattr(self, "expert_dp_group", None)
        if ep_dp is not None and dist.get_world_size(ep_dp) > 1:
            dist.all_reduce(self.grad_flat[self.model.dense_numel:], group=ep_dp)
