"""Qwen3-family decoder (dense and MoE) on the sm_100a kernel library.

One module serves both the trainer and the rollout engine:
  * `forward_train`   packed variable-length micro-batch (thd layout), optional per-layer
                      activation recompute, optional Rollout Routing Replay (R3)
  * `forward_prefill` packed prompts, writes K/V into the paged cache
  * `forward_decode`  one token per sequence against the paged cache
All three run the same kernels with the same reduction orders, so the log-prob of a token
computed in training is bitwise equal to the one the engine reported when it sampled it.

Parameters live in ONE flat bf16 buffer (`self.flat`) with named views; gradients accumulate
in a matching flat buffer (`main_grad` views) allocated by the trainer. The flat layout makes
the optimizer a single fused launch, and offload / refit a handful of large copies.

Reference: the GPT/MoE layer specs the reference builds through Megatron + TE
(megatron_utils/model_provider.py:27-250) and HF Qwen3 / Qwen3-MoE modelling.
"""
from __future__ import annotations

import collections

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from miles_b200.models.config import ModelConfig
from miles_b200.ops import gemm as G
from miles_b200.utils import dumper as _dumper
from miles_b200.ops.attention import PAGE, VarlenMeta, decode_attention, varlen_attention
from miles_b200.ops.moe import RouterCfg, emit_record, moe_experts
from miles_b200.ops.norm import (add_rms_norm, qk_norm_rope, qk_norm_rope_to_cache, rms_norm,
                                 rope_tables, swiglu)
from miles_b200.parallel.tp import (copy_to_tp, reduce_from_tp, row_parallel_rs, sp_gather,
                                    sp_gather_replicated, sp_reduce_scatter, sp_split)


@dataclass
class ParamSpec:
    name: str
    shape: tuple
    init: str  # "normal" | "ones" | "zeros"
    offset: int = 0

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


def param_specs(cfg: ModelConfig, ep_size: int = 1, tp_size: int = 1, layers=None,
                first: bool = True, last: bool = True, expert_tp: int | None = None) -> list[ParamSpec]:
    """Parameter layout; with expert parallelism each rank holds E / ep_size experts, with
    tensor parallelism each rank holds 1 / tp_size of the heads and intermediate dimensions
    (miles_b200/parallel/tp.py); a pipeline stage holds `layers` only, the embedding on the first
    stage and the final norm + LM head on the last (tied embeddings: a copy on the last stage).
    Routed experts split their intermediate dimension over `expert_tp` ranks (default: TP)."""
    H, D = cfg.hidden_size, cfg.head_dim
    t = tp_size
    if cfg.num_heads % t or cfg.num_kv_heads % t:
        raise ValueError(f"heads ({cfg.num_heads} q / {cfg.num_kv_heads} kv) do not split over TP {t}")
    nq, nkv = cfg.num_heads // t, cfg.num_kv_heads // t
    layers = range(cfg.num_layers) if layers is None else layers
    specs = []
    if first or (last and cfg.tie_embeddings):
        specs.append(ParamSpec("embed_tokens.weight", (cfg.vocab_size, H), "normal"))
    # multi-token prediction layers (on the last stage): ordinary decoder layers numbered after
    # the main stack, plus their input norms / projection and head norm (HF DeepSeek-V3 names)
    mtp_ids = list(range(cfg.num_layers, cfg.num_layers + cfg.mtp_num_layers)) if last else []
    for i in list(layers) + mtp_ids:
        p = f"layers.{i}."
        specs.append(ParamSpec(p + "input_layernorm.weight", (H,), "ones"))
        if cfg.layer_is_linear(i):  # Gated DeltaNet linear attention (models/gdn.py)
            from miles_b200.models.gdn import gdn_param_shapes

            specs += [ParamSpec(n, shp, init) for n, shp, init in gdn_param_shapes(cfg, p + "linear_attn.", t)]
        elif cfg.uses_torch_attention:  # gated / biased / partial-rotary attention (models/qwen3_next.py)
            from miles_b200.models.qwen3_next import gated_attn_param_shapes

            specs += [ParamSpec(n, shp, init) for n, shp, init in gated_attn_param_shapes(cfg, p + "self_attn.", t)]
        elif cfg.kv_lora_rank:  # multi-head latent attention (models/mla.py)
            from miles_b200.models.mla import mla_param_shapes

            specs += [ParamSpec(n, shp, init) for n, shp, init in mla_param_shapes(cfg, p + "self_attn.", t)]
        else:
            specs += [ParamSpec(p + "self_attn.qkv_proj.weight", ((nq + 2 * nkv) * D, H), "normal"),
                      ParamSpec(p + "self_attn.o_proj.weight", (H, nq * D), "normal")]
        specs.append(ParamSpec(p + "post_attention_layernorm.weight", (H,), "ones"))
        if cfg.sandwich_norm:  # GLM-4: norms on the attention and MLP outputs too
            specs += [ParamSpec(p + "post_self_attn_layernorm.weight", (H,), "ones"),
                      ParamSpec(p + "post_mlp_layernorm.weight", (H,), "ones")]
        if cfg.qk_norm and not cfg.kv_lora_rank and not cfg.layer_is_linear(i):
            specs += [ParamSpec(p + "self_attn.q_norm.weight", (D,), "ones"),
                      ParamSpec(p + "self_attn.k_norm.weight", (D,), "ones")]
        if cfg.layer_is_moe(i):
            E, I = cfg.num_experts, cfg.moe_intermediate_size // (t if expert_tp is None else expert_tp)
            El = E // ep_size
            specs += [ParamSpec(p + "mlp.gate.weight", (E, H), "normal"),
                      ParamSpec(p + "mlp.experts.w1", (El, 2 * I, H), "normal"),
                      ParamSpec(p + "mlp.experts.w2", (El, H, I), "normal")]
            if cfg.router_score == "sigmoid":
                specs.append(ParamSpec(p + "mlp.gate.e_score_correction_bias", (E,), "zeros"))
            if cfg.shared_expert_intermediate_size:  # Qwen3-Next: one gated shared expert
                Is = cfg.shared_expert_intermediate_size // t
                specs += [ParamSpec(p + "mlp.shared_expert.gate_up_proj.weight", (2 * Is, H), "normal"),
                          ParamSpec(p + "mlp.shared_expert.down_proj.weight", (H, Is), "normal"),
                          ParamSpec(p + "mlp.shared_expert_gate.weight", (1, H), "normal")]
            if cfg.num_shared_experts:
                Is = cfg.moe_intermediate_size * cfg.num_shared_experts // t
                specs += [ParamSpec(p + "mlp.shared_experts.gate_up_proj.weight", (2 * Is, H), "normal"),
                          ParamSpec(p + "mlp.shared_experts.down_proj.weight", (H, Is), "normal")]
        else:
            I = cfg.intermediate_size // t
            specs += [ParamSpec(p + "mlp.gate_up_proj.weight", (2 * I, H), "normal"),
                      ParamSpec(p + "mlp.down_proj.weight", (H, I), "normal")]
    for i in mtp_ids:
        p = f"layers.{i}."
        specs += [ParamSpec(p + "enorm.weight", (H,), "ones"), ParamSpec(p + "hnorm.weight", (H,), "ones"),
                  ParamSpec(p + "eh_proj.weight", (H, 2 * H), "normal"),
                  ParamSpec(p + "shared_head.norm.weight", (H,), "ones")]
    if last:
        specs.append(ParamSpec("norm.weight", (H,), "ones"))
        if not cfg.tie_embeddings:
            specs.append(ParamSpec("lm_head.weight", (cfg.vocab_size, H), "normal"))
    # Replicated (dense) parameters first, routed-expert parameters last: under expert
    # parallelism the two regions reduce over different groups.
    specs = [s for s in specs if not is_expert_param(s.name)] + [s for s in specs if is_expert_param(s.name)]
    off = 0
    for s in specs:
        s.offset = off
        off += (s.numel + 127) // 128 * 128  # 256-byte aligned views (TMA wants 16)
    return specs


def is_expert_param(name: str) -> bool:
    return ".mlp.experts." in name


FLAT_ALIGN = 8192


def kv_cache_shape(cfg: ModelConfig, tp_size: int = 1) -> tuple[int, int]:
    """(heads, dim) of one cached token per layer: GQA K and V (this TP rank's KV heads), or the
    MLA latent [c | k_pe] (replicated over TP ranks)."""
    if cfg.kv_lora_rank:  # + the DSA indexer key when the model has one
        return 1, cfg.kv_lora_rank + cfg.qk_rope_head_dim + (cfg.index_head_dim if cfg.index_topk else 0)
    return cfg.num_kv_heads // tp_size, cfg.head_dim


class KVCache:
    """Paged KV cache: per layer K and V of [num_pages * 64, nkv, 128] bf16.

    Zero-initialised: the decode kernel reads whole 128-key blocks, and slots past a sequence's
    context are masked out of the softmax but still multiplied (by zero) in the P.V product, so
    they must hold finite values."""

    def __init__(self, cfg: ModelConfig, num_pages: int, device, dtype=torch.bfloat16,
                 tp_size: int = 1, max_seqs: int = 0, buffer: torch.Tensor | None = None):
        """buffer: optional flat uint8 device tensor of at least `required_bytes(...)` that
        backs every cache tensor (e.g. a fixed-address arena); it is zeroed here."""
        self.num_pages = num_pages
        shapes = self.tensor_shapes(cfg, num_pages, tp_size, max_seqs, dtype)
        if buffer is not None:
            buffer.zero_()
            out, off = [], 0
            for shape, dt in shapes:
                n = math.prod(shape) * torch.empty((), dtype=dt).element_size()
                out.append(buffer[off:off + n].view(dt).view(shape) if n else
                           torch.zeros(shape, dtype=dt, device=device))
                off = (off + n + 255) // 256 * 256
        else:
            out = [torch.zeros(shape, dtype=dt, device=device) for shape, dt in shapes]
        L = cfg.num_layers
        self.k, self.v = out[:L], out[L:2 * L]
        # linear-attention layers: conv + recurrent state per engine batch slot (fp32)
        lin = [cfg.layer_is_linear(i) for i in range(L)]
        rest = iter(out[2 * L:])
        self.lin_conv, self.lin_state = [None] * L, [None] * L
        for i in range(L):
            if lin[i]:
                self.lin_conv[i], self.lin_state[i] = next(rest), next(rest)

    @staticmethod
    def tensor_shapes(cfg: ModelConfig, num_pages: int, tp_size: int = 1, max_seqs: int = 0,
                      dtype=torch.bfloat16) -> list:
        """[(shape, dtype)] of K per layer, V per layer, then (conv, state) per linear layer."""
        slots = num_pages * PAGE
        nkv, hd = kv_cache_shape(cfg, tp_size)
        lin = [cfg.layer_is_linear(i) for i in range(cfg.num_layers)]
        ks = [((0 if lin[i] else slots, nkv, hd), dtype) for i in range(cfg.num_layers)]
        # MLA caches only the latent (+ rotary key) in `k`
        vs = 1 if cfg.kv_lora_rank else slots
        vv = [((0 if lin[i] else vs, nkv, hd), dtype) for i in range(cfg.num_layers)]
        extra = []
        if any(lin):
            from miles_b200.models.gdn import gdn_state_shapes

            cs, ss = gdn_state_shapes(cfg, tp_size)
            for i in range(cfg.num_layers):
                if lin[i]:
                    extra += [((max_seqs,) + cs, torch.float32), ((max_seqs,) + ss, torch.float32)]
        return ks + vv + extra

    @classmethod
    def required_bytes(cls, cfg: ModelConfig, num_pages: int, tp_size: int = 1, max_seqs: int = 0,
                       dtype=torch.bfloat16) -> int:
        off = 0
        for shape, dt in cls.tensor_shapes(cfg, num_pages, tp_size, max_seqs, dtype):
            n = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            off = (off + n + 255) // 256 * 256
        return off

    def nbytes(self) -> int:
        ts = self.k + self.v + [t for t in self.lin_conv + self.lin_state if t is not None]
        return sum(t.numel() * t.element_size() for t in ts)


def dist_world(group) -> int:
    import torch.distributed as dist

    return dist.get_world_size(group)


class Transformer(torch.nn.Module):
    def __init__(self, cfg: ModelConfig, device="cuda", dtype=torch.bfloat16, seed: int = 0,
                 init_std: float = 0.02, materialize: bool = True, ep_group=None, tp_group=None,
                 tp_backend: str = "auto", tp_cap_rows: int = 16384, cp_group=None,
                 pp_group=None, ep_cap_tokens: int = 16384, vpp: int = 1,
                 pp_first_layers: int | None = None, pp_last_layers: int | None = None,
                 etp: int | None = None):
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.tp = None
        if tp_group is not None:
            from miles_b200.parallel.tp import TPContext

            self.tp = TPContext(tp_group, tp_backend, cfg.hidden_size, tp_cap_rows)
            if self.tp.size == 1:
                self.tp = None
        self.tp_size = self.tp.size if self.tp else 1
        # sequence parallelism (training forward): residual stream sharded over TP ranks by rows
        self.sequence_parallel = False
        # TP trainer log-probs with the vocabulary split over the TP ranks (opt-in: the rollout
        # engine samples from full logits, so train / rollout log-probs then differ by rounding)
        self.vocab_parallel_logprob = False
        self.cp = None  # context parallelism (training forward), miles_b200/parallel/cp.py
        if cp_group is not None:
            from miles_b200.parallel.cp import CPContext

            self.cp = CPContext(cp_group)
            if self.cp.size == 1:
                self.cp = None
            else:
                nq_l, nkv_l, c = cfg.num_heads // self.tp_size, cfg.num_kv_heads // self.tp_size, self.cp.size
                if nq_l % c or (nkv_l % c and c % nkv_l):
                    raise ValueError(f"{nq_l} q / {nkv_l} KV heads per TP rank do not split over "
                                     f"CP {c} (KV heads must split over it or divide it)")
        self.nq = cfg.num_heads // self.tp_size      # this rank's query heads
        self.nkv = cfg.num_kv_heads // self.tp_size  # this rank's KV heads
        self.ep = None
        if ep_group is not None and cfg.is_moe:
            from miles_b200.parallel.ep import EPContext

            self.ep = EPContext(ep_group, cfg.num_experts, "auto", cfg.hidden_size, cfg.topk,
                                cap_tokens=ep_cap_tokens)
            if self.ep.size == 1:
                self.ep = None
        self.pp = None  # pipeline parallelism (training), miles_b200/parallel/pp.py
        if pp_group is not None:
            from miles_b200.parallel.pp import PPContext

            self.pp = PPContext(pp_group, cfg.num_layers, vpp, pp_first_layers, pp_last_layers)
            if self.pp.size == 1:
                self.pp = None
            elif self.tp is not None or self.cp is not None or self.ep is not None:
                raise ValueError("pipeline parallelism is supported with data parallelism only")
        self.layer_ids = list(self.pp.layer_ids) if self.pp else list(range(cfg.num_layers))
        self.mtp_ids = list(range(cfg.num_layers, cfg.num_layers + cfg.mtp_num_layers))
        if self.mtp_ids and (self.pp is not None or self.tp is not None or self.cp is not None
                             or self.ep is not None):
            raise ValueError("multi-token prediction layers run with data parallelism only")
        if self.mtp_ids and cfg.linear_attn_interval > 0:
            # Qwen3-Next / Qwen3.5 keep their MTP block under mtp.fc / mtp.pre_fc_norm_* with
            # gated full attention; that layout is not mapped here
            raise ValueError("multi-token prediction is not supported on Gated DeltaNet hybrid "
                             "families (Qwen3-Next / Qwen3.5)")
        self.mtp_train = False  # add the MTP loss in training (Actor)
        self._mtp_h = None
        self.is_first = self.pp is None or self.pp.is_first
        self.is_last = self.pp is None or self.pp.is_last
        # expert-tensor parallelism: routed experts split over the TP ranks (etp = TP, default)
        # or whole on every rank (etp = 1: each TP rank routes its 1 / TP of the tokens)
        if etp not in (None, 1, self.tp_size):
            raise ValueError(f"expert-tensor-parallel size {etp} must be 1 or the TP size {self.tp_size}")
        self.expert_tp = self.tp_size if etp is None else etp
        self.specs = param_specs(cfg, self.ep.size if self.ep else 1, self.tp_size, self.layer_ids,
                                 self.is_first, self.is_last, self.expert_tp)
        total = self.specs[-1].offset + self.specs[-1].numel
        self.numel = total
        ex = [sp.offset for sp in self.specs if is_expert_param(sp.name)]
        self.dense_numel = ex[0] if ex else total
        # padded to a multiple of 8192 elements so that the flat buffers split evenly over
        # 1/2/4/8 data-parallel ranks (sharded optimizer); the tail is never a parameter
        padded = (total + FLAT_ALIGN - 1) // FLAT_ALIGN * FLAT_ALIGN
        self.flat = torch.zeros(padded, dtype=dtype, device=self.device) if padded != total else \
            torch.empty(total, dtype=dtype, device=self.device)
        self.params: dict[str, torch.nn.Parameter] = {}
        for s in self.specs:
            p = torch.nn.Parameter(self.flat[s.offset:s.offset + s.numel].view(s.shape))
            self.params[s.name] = p
        if materialize:
            self.init_weights(seed, init_std)
            if self.pp is not None and cfg.tie_embeddings:
                from miles_b200.parallel.pp import sync_tied_embedding

                sync_tied_embedding(self)
        self.rope_cos, self.rope_sin = rope_tables(cfg.max_position, cfg.head_dim, cfg.rope_theta,
                                                   self.device, cfg.rope_scaling)
        self.router_cfgs = {}
        if cfg.is_moe:
            rc = RouterCfg(cfg.num_experts, cfg.topk, cfg.router_score, cfg.norm_topk_prob,
                           cfg.n_group, cfg.topk_group, cfg.routed_scaling_factor)
            for i in self.layer_ids + self.mtp_ids:
                if cfg.layer_is_moe(i):
                    self.router_cfgs[i] = rc
        # global ordinal of every MoE layer (column of the R3 routing tensors)
        self.moe_index = {i: j for j, i in enumerate(i for i in range(cfg.num_layers) if cfg.layer_is_moe(i))}
        self.recompute = True
        self.weight_version = 0
        self.fp8: dict = {}  # name -> Fp8Weight (block-scaled fp8 copies, see enable_fp8)
        self._fp8_version = None
        self.fp8_sync_events = collections.deque(maxlen=256)
        # fp32 pinning (the reference's mark_param_dtype): parameters whose runtime value stays
        # fp32 although the flat buffer is bf16 (see pinned_param)
        self.fp32 = {n: p.detach().float().clone() for n, p in self.params.items()
                     if n.endswith(self.FP32_PINNED)}
        self._fp32_snap = {n: p.detach().clone() for n, p in self.params.items() if n in self.fp32}
        self._fp32_version = self.weight_version
        self.qat: dict = {}  # name -> fake-int4 weight value (int4 quantisation-aware training)
        self.qat_group = 128
        self._qat_version = None
        self.lora = None  # miles_b200.models.lora.LoRA when adapters are attached
        self.gdn = None
        if cfg.linear_attn_interval:
            from miles_b200.models.gdn import GDN

            self.gdn = GDN(self)
        self.gattn = None
        if cfg.uses_torch_attention and not cfg.kv_lora_rank:
            from miles_b200.models.qwen3_next import GatedAttention

            self.gattn = GatedAttention(self)
        self.mla = None
        if cfg.kv_lora_rank:
            from miles_b200.models.mla import MLA

            self.mla = MLA(self)

    # -------------------------------------------------------------------------------- projections
    def _lin(self, x: torch.Tensor, name: str) -> torch.Tensor:
        y = G.linear(x, self.params[name])
        if self.lora is not None and name in self.lora:
            y = y + self.lora.delta(name, x)
        return y

    def _lin_swiglu(self, x: torch.Tensor, name: str) -> torch.Tensor:
        if self.lora is not None and name in self.lora:
            return swiglu(self._lin(x, name))
        return G.linear_swiglu(x, self.params[name])

    # -------------------------------------------------------------------------------- fp32 pinning
    FP32_PINNED = ("mlp.gate.e_score_correction_bias", "linear_attn.A_log", "linear_attn.dt_bias")

    def pinned_param(self, name: str):
        """The runtime value of parameter `name`: for the fp32-pinned parameters (the router's
        expert-score bias, Gated DeltaNet's A_log / dt_bias) the fp32 copy, which keeps what a
        checkpoint stored in fp32; gradients still reach the bf16 parameter (straight through)."""
        p = self.params.get(name)
        f = self.fp32.get(name)
        if p is None or f is None:
            return p
        if torch.is_grad_enabled() and p.requires_grad:
            return f + (p - p.detach()).float()
        return f

    @torch.no_grad()
    def _sync_fp32(self) -> None:
        """After a weight update (new version) a pinned parameter whose bf16 value changed takes
        that value; unchanged ones keep their fp32 value. Not inside a CUDA graph capture."""
        if not self.fp32 or self._fp32_version == self.weight_version:
            return
        if self.device.type == "cuda" and torch.cuda.is_current_stream_capturing():
            return
        for n, f in self.fp32.items():
            p = self.params[n].data
            if not torch.equal(p, self._fp32_snap[n]):
                f.copy_(p.float())
                self._fp32_snap[n].copy_(p)
        self._fp32_version = self.weight_version

    @torch.no_grad()
    def set_fp32_value(self, name: str, value: torch.Tensor) -> None:
        """Load a full-precision value for a pinned parameter (checkpoint loaders)."""
        if name in self.fp32:
            self.fp32[name].copy_(value.float())
            self.params[name].data.copy_(value.to(self.params[name].dtype))
            self._fp32_snap[name].copy_(self.params[name].data)

    # -------------------------------------------------------------------------------- fp8
    FP8_SUFFIXES = ("qkv_proj.weight", "o_proj.weight", "gate_up_proj.weight", "down_proj.weight",
                    "q_proj.weight", "k_proj.weight", "v_proj.weight", "experts.w1", "experts.w2")

    def enable_fp8(self) -> None:
        """Unified block-scaled fp8 (the reference's `--fp8-format e4m3 --fp8-recipe
        blockwise` training with fp8 rollout): every linear / grouped-expert weight gets an e4m3
        copy with 128 x 128 block scales, and the forward GEMMs of training, prefill and decode
        run on it (activations quantised 1 x 128 on the fly). Training and rollout use the same
        copy and the same kernels, so their log-probs stay bitwise equal. The bf16 parameters
        stay the master copy: the backward uses them and the optimizer updates them; the fp8
        copy is re-quantised in place (same addresses, so decode graphs stay valid) whenever the
        weight version changes. Embeddings, the LM head, the router and norms stay bf16, as in
        the reference."""
        from miles_b200.ops.fp8 import Fp8Weight, register_fp8

        if self.tp is not None or self.lora is not None:
            raise ValueError("block-scaled fp8 GEMMs run without tensor parallelism and LoRA")
        for name, p in self.params.items():
            if not name.endswith(self.FP8_SUFFIXES) or p.dim() < 2:
                continue
            if p.shape[-1] % 128 or (p.numel() // p.shape[-1]) % 128:
                continue
            w8 = Fp8Weight.empty_like(p)
            register_fp8(p, w8)
            self.fp8[name] = w8
        self.sync_fp8(force=True)

    def enable_int4_qat(self, group: int = 128) -> None:
        """Int4 quantisation-aware training of the routed experts (the reference's
        OPEN_TRAINING_INT4_FAKE_QAT_FLAG / OPEN_TRAINING_INT4_GROUP_SIZE): the expert GEMMs of
        training, prefill and decode use the fake-int4 value of each expert weight (symmetric
        int4 in groups of `group` along K, re-computed whenever the weight version changes),
        the data-gradient uses it too, and the weight-gradient goes straight through to the bf16
        weight (straight-through estimator). The rollout engine therefore runs the int4-rounded
        experts the training forward sees, like an int4 (W4A16) rollout."""
        if self.fp8:
            raise ValueError("int4 QAT and block fp8 are exclusive")
        self.qat_group = group
        for name, p in self.params.items():
            if name.endswith(("experts.w1", "experts.w2")):
                self.qat[name] = torch.empty_like(p.data)
        self._qat_version = None
        self.sync_fp8()

    def expert_weight(self, name: str) -> torch.Tensor:
        """The tensor the expert GEMMs use for parameter `name` (its fake-int4 value under QAT).
        On the kernel path the fake-int4 copy shares the parameter's gradient buffer, so the
        weight-gradient GEMM accumulates into it (straight-through); the PyTorch path builds the
        same estimator with autograd."""
        p = self.params[name]
        q = self.qat.get(name)
        if q is None:
            return p
        if not G.use_native(q):
            return p + (q - p).detach()
        g = G.main_grad_of(p)
        if g is not None:
            G.register_main_grad(q, g)
        return q

    def disable_fp8(self) -> None:
        from miles_b200.ops.fp8 import unregister_fp8

        for name in self.fp8:
            unregister_fp8(self.params[name])
        self.fp8 = {}

    @torch.no_grad()
    def sync_fp8(self, force: bool = False) -> None:
        """Re-quantise the fp8 copies when the bf16 weights changed (new weight version); not
        inside a CUDA graph capture (the captured kernels read the copies in place). Also
        refreshes the int4-QAT values and the fp32-pinned parameters."""
        self._sync_fp32()
        if self.qat and self._qat_version != self.weight_version and not (
                self.device.type == "cuda" and torch.cuda.is_current_stream_capturing()):
            from miles_b200.ops.quant import int4_qat_weight

            for name, q in self.qat.items():
                int4_qat_weight(self.params[name].data, self.qat_group, out=q)
            self._qat_version = self.weight_version
        if not self.fp8 or (not force and self._fp8_version == self.weight_version):
            return
        if self.device.type == "cuda" and torch.cuda.is_current_stream_capturing():
            return
        ev = None
        if self.device.type == "cuda":
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        for name, w8 in self.fp8.items():
            w8.requant_(self.params[name])
        if ev is not None:
            ev[1].record()
            self.fp8_sync_events.append(ev)  # device time of each re-quantisation (refit)
        self._fp8_version = self.weight_version

    # -------------------------------------------------------------------------------- params
    @torch.no_grad()
    def init_weights(self, seed: int, std: float):
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        chunk = 1 << 26
        for s in self.specs:
            t = self.flat[s.offset:s.offset + s.numel]
            if s.init == "ones":
                t.fill_(1.0)
            elif s.init == "zeros":
                t.zero_()
            else:
                for a in range(0, s.numel, chunk):
                    b = min(s.numel, a + chunk)
                    t[a:b] = (torch.randn(b - a, generator=g, device=self.device) * std).to(self.dtype)

    def named_flat_params(self):
        return self.params.items()

    def p(self, name: str) -> torch.Tensor:
        return self.params[name]

    def lm_head_weight(self) -> torch.Tensor:
        return self.params["embed_tokens.weight" if self.cfg.tie_embeddings else "lm_head.weight"]

    # -------------------------------------------------------------------------------- blocks
    def _attn_train(self, i: int, x: torch.Tensor, meta: VarlenMeta) -> torch.Tensor:
        return self._sw(i, "post_self_attn_layernorm", self._attn_train_raw(i, x, meta))

    def _attn_train_raw(self, i: int, x: torch.Tensor, meta: VarlenMeta) -> torch.Tensor:
        cfg = self.cfg
        if self.gdn is not None and cfg.layer_is_linear(i):
            return self.gdn.attn(i, x, meta)
        if self.gattn is not None:
            return self.gattn.attn(i, x, meta)
        if self.mla is not None:
            return self.mla.attn(i, x, meta)
        pre = f"layers.{i}.self_attn."
        qkv = self._lin(copy_to_tp(x, self.tp), pre + "qkv_proj.weight")
        q, k, v = qk_norm_rope(qkv, self.params.get(pre + "q_norm.weight"),
                               self.params.get(pre + "k_norm.weight"), meta.positions,
                               self.rope_cos, self.rope_sin, self.nq, self.nkv,
                               cfg.rms_eps, cfg.qk_norm)
        o = varlen_attention(q, k, v, meta)
        return reduce_from_tp(self._lin(o.reshape(x.shape[0], -1), pre + "o_proj.weight"), self.tp)

    def _sw(self, i: int, name: str, t):
        """GLM-4 sandwich norm of a branch output (identity for other families)."""
        if not self.cfg.sandwich_norm:
            return t
        return rms_norm(t, self.params[f"layers.{i}.{name}.weight"], self.cfg.rms_eps)

    def _mlp(self, i: int, x: torch.Tensor, replay=None, record=None) -> torch.Tensor:
        m = reduce_from_tp(self._mlp_partial(i, copy_to_tp(x, self.tp), replay, record), self.tp)
        return self._sw(i, "post_mlp_layernorm", m)

    def _mlp_partial(self, i: int, x: torch.Tensor, replay=None, record=None) -> torch.Tensor:
        """MLP / MoE output before the tensor-parallel all-reduce (the full output at TP 1)."""
        pre = f"layers.{i}.mlp."
        if i in self.router_cfgs:
            y = self._routed(i, x, replay, record)
            if self.cfg.num_shared_experts:
                s = G.linear_swiglu(x, self.params[pre + "shared_experts.gate_up_proj.weight"])
                y = y + G.linear(s, self.params[pre + "shared_experts.down_proj.weight"])
            if self.cfg.shared_expert_intermediate_size:
                s = G.linear_swiglu(x, self.params[pre + "shared_expert.gate_up_proj.weight"])
                gate = torch.sigmoid((x.float() @ self.params[pre + "shared_expert_gate.weight"].float().t()))
                y = y + (gate * G.linear(s, self.params[pre + "shared_expert.down_proj.weight"]).float()).to(y.dtype)
            return y
        return self._lin(self._lin_swiglu(x, pre + "gate_up_proj.weight"), pre + "down_proj.weight")

    def _routed(self, i: int, x: torch.Tensor, replay=None, record=None) -> torch.Tensor:
        """Routed experts of layer i. With whole experts under TP (expert_tp = 1) each TP rank
        routes rows [T r / tp, T (r+1) / tp) of the replicated input and returns them in a
        zero-filled [T, H] block, so the TP all-reduce that follows completes the output (and
        the backward of the TP copy sums the row gradients)."""
        pre = f"layers.{i}.mlp."
        args = (self.params[pre + "gate.weight"], self.expert_weight(pre + "experts.w1"),
                self.expert_weight(pre + "experts.w2"), self.router_cfgs[i])
        bias = self.pinned_param(pre + "gate.e_score_correction_bias")

        def run(xr, rp, rec):
            if self.ep is not None:
                from miles_b200.parallel.ep import moe_experts_ep

                return moe_experts_ep(xr, *args, self.ep, bias, rp, rec)
            return moe_experts(xr, *args, bias, rp, rec)

        if self.tp is None or self.expert_tp > 1:
            return run(x, replay, record)
        T, tp = x.shape[0], self.tp
        lo, hi = T * tp.rank // tp.size, T * (tp.rank + 1) // tp.size
        got = []
        y = run(x[lo:hi], None if replay is None else replay[lo:hi],
                None if record is None else got.append)
        if record is not None:  # the full routing: every rank's rows, gathered
            idx = got[0]
            n = -(-T // tp.size) + 1
            buf = torch.full((n, idx.shape[1]), -1, dtype=idx.dtype, device=idx.device)
            buf[:hi - lo] = idx
            parts = [torch.empty_like(buf) for _ in range(tp.size)]
            dist.all_gather(parts, buf, group=tp.group)
            emit_record(record, torch.cat([p[:(T * (r + 1) // tp.size) - (T * r // tp.size)]
                                           for r, p in enumerate(parts)], 0))
        return F.pad(y, (0, 0, lo, T - hi))

    def _layer_train(self, i, m_prev, r_prev, meta, replay):
        cfg = self.cfg
        ln1 = self.params[f"layers.{i}.input_layernorm.weight"]
        if m_prev is None:
            x, r = rms_norm(r_prev, ln1, cfg.rms_eps), r_prev
        else:
            x, r = add_rms_norm(m_prev, r_prev, ln1, cfg.rms_eps)
        a = self._attn_train(i, x, meta)
        x2, r = add_rms_norm(a, r, self.params[f"layers.{i}.post_attention_layernorm.weight"],
                             cfg.rms_eps)
        m = self._mlp(i, x2, replay=replay)
        return m, r

    # -------------------------------------------------------------------------------- layer loop
    def _run_layers(self, layer_fn, r, replay_experts, rows=None, layers=None):
        """Run this rank's layers: layer_fn(i, m_prev, r_prev, replay) -> (m, r), with per-layer
        activation recompute when training. `replay_experts` [T, L_moe, k] is sliced to layer i's
        MoE column (and to `rows`, a slice of this rank's rows, if given)."""
        m = None
        rc_limit = getattr(self, "recompute_layers", None)  # recompute only the first N (block)
        for li, i in enumerate(self.layer_ids if layers is None else layers):
            replay = None
            if i in self.router_cfgs and replay_experts is not None:
                col = replay_experts[:, self.moe_index[i]]
                replay = (col if rows is None else col[rows]).contiguous()
            # layers that exchange point-to-point messages in their forward (linear attention
            # under CP) are not recomputed: a recompute would send the messages twice
            p2p = self.cp is not None and self.cfg.layer_is_linear(i)
            if (self.recompute and torch.is_grad_enabled() and not p2p
                    and (rc_limit is None or li < rc_limit)):
                if m is None:
                    m, r = checkpoint(lambda rr, i=i, rp=replay: layer_fn(i, None, rr, rp), r,
                                      use_reentrant=False)
                else:
                    m, r = checkpoint(lambda mm, rr, i=i, rp=replay: layer_fn(i, mm, rr, rp), m, r,
                                      use_reentrant=False)
            else:
                m, r = layer_fn(i, m, r, replay)
        return m, r

    # -------------------------------------------------------------------------------- sequence parallel
    def _layer_train_sp(self, i, m_prev, r_prev, meta, replay):
        """One layer on this rank's rows: norms on T/tp rows, column-parallel projections on the
        all-gathered rows, row-parallel projections ending in a (fused) reduce-scatter."""
        cfg, tp = self.cfg, self.tp
        ln1 = self.params[f"layers.{i}.input_layernorm.weight"]
        if m_prev is None:
            x, r = rms_norm(r_prev, ln1, cfg.rms_eps), r_prev
        else:
            x, r = add_rms_norm(m_prev, r_prev, ln1, cfg.rms_eps)
        pre = f"layers.{i}.self_attn."
        if self.gdn is not None and cfg.layer_is_linear(i):  # Gated DeltaNet (models/gdn.py)
            a = self.gdn.attn_sp(i, x, meta)
        elif self.mla is not None:  # latents gathered instead of the hidden rows (models/mla.py)
            a = self.mla.attn_sp(i, x, meta)
        elif self.gattn is not None:  # separate q / k / v (models/qwen3_next.py)
            a = self.gattn.attn_sp(i, x, meta)
        else:
            xf = sp_gather(x, tp)
            qkv = self._lin(xf, pre + "qkv_proj.weight")
            q, k, v = qk_norm_rope(qkv, self.params.get(pre + "q_norm.weight"),
                                   self.params.get(pre + "k_norm.weight"), meta.positions,
                                   self.rope_cos, self.rope_sin, self.nq, self.nkv, cfg.rms_eps, cfg.qk_norm)
            o = varlen_attention(q, k, v, meta)
            a = self._row_rs(o.reshape(xf.shape[0], -1), pre + "o_proj.weight")
        # GLM-4 sandwich norms act row by row: on this rank's rows after the reduce-scatter
        a = self._sw(i, "post_self_attn_layernorm", a)
        x2, r = add_rms_norm(a, r, self.params[f"layers.{i}.post_attention_layernorm.weight"], cfg.rms_eps)
        x2f = sp_gather(x2, tp)
        if i in self.router_cfgs:
            m = sp_reduce_scatter(self._mlp_partial(i, x2f, replay=replay), tp)
        else:
            pm = f"layers.{i}.mlp."
            m = self._row_rs(self._lin_swiglu(x2f, pm + "gate_up_proj.weight"), pm + "down_proj.weight")
        return self._sw(i, "post_mlp_layernorm", m), r

    def _row_rs(self, a: torch.Tensor, name: str) -> torch.Tensor:
        if self.lora is not None and name in self.lora:
            return sp_reduce_scatter(self._lin(a, name), self.tp)
        return row_parallel_rs(a, self.params[name], self.tp, G.linear)

    def _forward_train_sp(self, tokens, meta, replay_experts):
        from miles_b200.ops.attention import VarlenMeta

        cfg, tp = self.cfg, self.tp
        T = tokens.shape[0]
        pad = (-T) % tp.size
        if pad:
            # a padding sequence at the end so the rows split evenly over the TP ranks
            tokens = torch.cat([tokens, tokens.new_zeros(pad)])
            meta = VarlenMeta(list(meta.cu_list) + [T + pad], tokens.device)
            if replay_experts is not None:
                replay_experts = torch.cat([replay_experts, replay_experts[:1].expand(pad, -1, -1)])
        r = sp_split(F.embedding(tokens.long(), self.params["embed_tokens.weight"]), tp)
        m, r = self._run_layers(lambda i, mm, rr, rp: self._layer_train_sp(i, mm, rr, meta, rp), r,
                                replay_experts)
        y, _ = add_rms_norm(m, r, self.params["norm.weight"], cfg.rms_eps)
        return sp_gather_replicated(y, tp)[:T]

    # -------------------------------------------------------------------------------- context parallel
    def _layer_train_cp(self, i, m_prev, r_prev, meta, pos, replay):
        cfg, cp = self.cfg, self.cp
        from miles_b200.parallel.cp import heads_to_tokens, kv_tokens_to_heads, tokens_to_heads

        ln1 = self.params[f"layers.{i}.input_layernorm.weight"]
        if m_prev is None:
            x, r = rms_norm(r_prev, ln1, cfg.rms_eps), r_prev
        else:
            x, r = add_rms_norm(m_prev, r_prev, ln1, cfg.rms_eps)
        if self.gdn is not None and cfg.layer_is_linear(i):
            # linear attention: state hand-over between consecutive CP ranks (models/gdn.py)
            from miles_b200.models.gdn import gdn_attn_cp

            _, lo, hi = cp.rows(meta.total)
            a = gdn_attn_cp(self.gdn, i, x, meta, lo, hi, cp)
            x2, r = add_rms_norm(self._sw(i, "post_self_attn_layernorm", a), r,
                                 self.params[f"layers.{i}.post_attention_layernorm.weight"], cfg.rms_eps)
            return self._mlp(i, x2, replay=replay), r
        pre = f"layers.{i}.self_attn."
        if self.mla is not None:  # multi-head latent attention (+ DSA): models/mla.py
            a = self.mla.attn_cp(i, x, meta, pos, cp)
            x2, r = add_rms_norm(a, r, self.params[f"layers.{i}.post_attention_layernorm.weight"],
                                 cfg.rms_eps)
            return self._mlp(i, x2, replay=replay), r
        if self.gattn is not None:  # gated attention (Qwen3-Next): same head exchange
            q, k, v, gate = self.gattn._qkv(i, x, pos)
            qh, kh, vh = tokens_to_heads(q, cp), kv_tokens_to_heads(k, cp), kv_tokens_to_heads(v, cp)
            if self.gattn._native(x):
                oh = varlen_attention(qh, kh, vh, meta)
            else:
                oh = self.gattn._sdpa(qh, kh, vh, meta.cu_list)
            a = self.gattn._out(i, heads_to_tokens(oh, cp), gate)
            x2, r = add_rms_norm(self._sw(i, "post_self_attn_layernorm", a), r,
                                 self.params[f"layers.{i}.post_attention_layernorm.weight"], cfg.rms_eps)
            return self._mlp(i, x2, replay=replay), r
        # under TP the projections hold this TP rank's heads; the CP exchange splits those
        qkv = self._lin(copy_to_tp(x, self.tp), pre + "qkv_proj.weight")
        q, k, v = qk_norm_rope(qkv, self.params.get(pre + "q_norm.weight"),
                               self.params.get(pre + "k_norm.weight"), pos,
                               self.rope_cos, self.rope_sin, self.nq, self.nkv, cfg.rms_eps, cfg.qk_norm)
        o = varlen_attention(tokens_to_heads(q, cp), kv_tokens_to_heads(k, cp), kv_tokens_to_heads(v, cp), meta)
        a = reduce_from_tp(self._lin(heads_to_tokens(o, cp).reshape(x.shape[0], -1), pre + "o_proj.weight"),
                           self.tp)
        x2, r = add_rms_norm(self._sw(i, "post_self_attn_layernorm", a), r,
                                 self.params[f"layers.{i}.post_attention_layernorm.weight"], cfg.rms_eps)
        return self._mlp(i, x2, replay=replay), r

    def _forward_train_cp(self, tokens, meta, replay_experts):
        """Final hidden of this CP rank's rows [lo, hi) of the (padded) batch."""
        from miles_b200.ops.attention import VarlenMeta

        cfg, cp = self.cfg, self.cp
        T = tokens.shape[0]
        Tp, lo, hi = cp.rows(T)
        if Tp > T:
            tokens = torch.cat([tokens, tokens.new_zeros(Tp - T)])
            meta = VarlenMeta(list(meta.cu_list) + [Tp], tokens.device)
            if replay_experts is not None:
                replay_experts = torch.cat([replay_experts, replay_experts[:1].expand(Tp - T, -1, -1)])
        pos = meta.positions[lo:hi].contiguous()
        r = F.embedding(tokens[lo:hi].long(), self.params["embed_tokens.weight"])
        m, r = self._run_layers(lambda i, mm, rr, rp: self._layer_train_cp(i, mm, rr, meta, pos, rp), r,
                                replay_experts, rows=slice(lo, hi))
        y, _ = add_rms_norm(m, r, self.params["norm.weight"], cfg.rms_eps)
        return y

    def mtp_loss(self, tokens, meta, sel, targets, weights, temperature: float = 1.0,
                 chunk: int = 4096) -> torch.Tensor:
        """Multi-token prediction loss of the last training forward (`selected_logprob` keeps
        its final hidden h). Depth k (1-based) at row t: layer num_layers + k - 1 over
        eh_proj([enorm(emb(token t + k)); hnorm(h_{k-1}[t])]) (the token embedding detached,
        h_0 = h), then the shared LM head after shared_head.norm predicts token t + k + 1. The
        main forward scores target tokens[s + 1] at rows `sel`; depth k scores the same targets
        at rows s - k of the same sequence. Returns the mean over depths of
        -sum(weights * log p) over the rows that exist.

        Reference: Megatron MTP block (model_provider.py, --enable-mtp-training, MTP loss scaled
        by --mtp-loss-scaling-factor), embeddings detached in the MTP input (megatron.patch)."""
        from miles_b200.ops.logprob import lm_head_logprob

        cfg = self.cfg
        h = self._mtp_h
        T = tokens.shape[0]
        dev = tokens.device
        cu = torch.tensor(meta.cu_list, device=dev)
        row = torch.arange(T, device=dev)
        seq = torch.searchsorted(cu, row, right=True) - 1
        start, end = cu[seq], cu[seq + 1]
        emb = F.embedding(tokens.long(), self.params["embed_tokens.weight"]).detach()
        W = self.lm_head_weight()
        prev, total = h, h.new_zeros((), dtype=torch.float32)
        for k, j in enumerate(self.mtp_ids, 1):
            p = f"layers.{j}."
            ahead = row + k
            ok = ahead < end
            e = emb[torch.where(ok, ahead, row)] * ok[:, None].to(emb.dtype)
            x = torch.cat([rms_norm(e, self.params[p + "enorm.weight"], cfg.rms_eps),
                           rms_norm(prev, self.params[p + "hnorm.weight"], cfg.rms_eps)], -1)
            x = self._lin(x, p + "eh_proj.weight")
            m, r = self._layer_train(j, None, x, meta, None)
            prev = m + r
            y = rms_norm(prev, self.params[p + "shared_head.norm.weight"], cfg.rms_eps)
            rows = sel - k
            valid = rows >= start[sel]
            rows = torch.where(valid, rows, sel)
            lp, _ = lm_head_logprob(y.index_select(0, rows), W, targets, temperature, chunk)
            total = total - (weights * valid.to(weights.dtype) * lp.float()).sum()
        return total / max(1, len(self.mtp_ids))

    def selected_logprob(self, tokens, meta, sel, targets, temperature: float, chunk: int,
                         replay_experts=None):
        """(log-prob, entropy) of `targets` at hidden rows `sel` (ascending) of the training
        forward. Under context parallelism each rank scores the rows it holds and the results
        are all-gathered; every CP rank returns the full vectors."""
        from miles_b200.ops.logprob import lm_head_logprob

        W = self.lm_head_weight()
        h = self.forward_train(tokens, meta, replay_experts=replay_experts)
        self._mtp_h = h if (self.mtp_train and torch.is_grad_enabled()) else None
        if self.tp is not None and self.vocab_parallel_logprob and self.cp is None:
            from miles_b200.parallel.tp import vocab_parallel_logprob

            if self.cfg.tie_embeddings:
                raise ValueError("vocab-parallel log-probs need an untied LM head")

            return vocab_parallel_logprob(h.index_select(0, sel), W, targets, temperature, self.tp, chunk)
        if self.cp is None:
            return lm_head_logprob(h.index_select(0, sel), W, targets, temperature, chunk)
        from miles_b200.parallel.cp import gather_parts

        cp = self.cp
        Tp, lo, hi = cp.rows(tokens.shape[0])
        R = hi - lo
        sel_h = sel.cpu()
        sizes = [int(((sel_h >= r * R) & (sel_h < (r + 1) * R)).sum()) for r in range(cp.size)]
        mask = (sel >= lo) & (sel < hi)
        idx = sel[mask] - lo
        if idx.numel():
            lp, ent = lm_head_logprob(h.index_select(0, idx), W, targets[mask], temperature, chunk)
        else:
            # nothing to score here; stay on the autograd graph so the backward (and its
            # collectives) runs on every CP rank
            z = (h[:1].float().sum() * 0).reshape(1)[:0]
            lp, ent = z, z
        return gather_parts(lp, cp, sizes), gather_parts(ent, cp, sizes)

    # -------------------------------------------------------------------------------- train
    def forward_train(self, tokens: torch.Tensor, meta: VarlenMeta,
                      replay_experts: torch.Tensor | None = None,
                      record_experts: list | None = None,
                      hidden_in: torch.Tensor | None = None, chunk: int | None = None) -> torch.Tensor:
        """tokens int [T] packed; returns final hidden [T, H] (after the final norm).
        replay_experts: int32 [T, L_moe, k] routing to replay (R3).
        Pipeline stages: a stage after the first takes the residual stream `hidden_in`, a stage
        before the last returns its residual stream (bitwise what the next layer's fused
        residual add would have formed). With interleaved stages (`vpp` > 1) `chunk` selects the
        model chunk to run: the embedding belongs to chunk 0 of the first rank, the final norm to
        the last chunk of the last rank."""
        cfg = self.cfg
        self.sync_fp8()
        if self.tp is not None and self.sequence_parallel and record_experts is None and self.cp is None:
            return self._forward_train_sp(tokens, meta, replay_experts)
        if self.cp is not None:
            if record_experts is not None:
                raise NotImplementedError("routing capture under context parallelism")
            return self._forward_train_cp(tokens, meta, replay_experts)
        layers, first, last = None, self.is_first, self.is_last
        if chunk is not None and self.pp is not None:
            lo, hi = self.pp.chunks[chunk]
            layers = list(range(lo, hi))
            first, last = first and chunk == 0, last and chunk == self.pp.vpp - 1
        r = F.embedding(tokens.long(), self.params["embed_tokens.weight"]) if first else hidden_in

        def layer(i, m, r, replay):
            if (record_experts is not None and i in self.router_cfgs
                    and not (self.recompute and torch.is_grad_enabled())):
                # routing capture (R3): the MoE call reports the routing it used
                ln1 = self.params[f"layers.{i}.input_layernorm.weight"]
                x, r = (rms_norm(r, ln1, cfg.rms_eps), r) if m is None else add_rms_norm(m, r, ln1, cfg.rms_eps)
                a = self._attn_train(i, x, meta)
                x2, r = add_rms_norm(a, r, self.params[f"layers.{i}.post_attention_layernorm.weight"], cfg.rms_eps)
                return self._mlp(i, x2, replay=replay, record=record_experts.append), r
            out = self._layer_train(i, m, r, meta, replay)
            if _dumper.enabled():  # per-layer residual stream (--dumper-enable)
                _dumper.dump(f"layer{i:03d}_residual", out[1])
            return out

        m, r = self._run_layers(layer, r, replay_experts, layers=layers)
        if not last:
            return r if m is None else m + r
        y, _ = add_rms_norm(m, r, self.params["norm.weight"], cfg.rms_eps)
        if _dumper.enabled():
            _dumper.dump("final_hidden", y)
        return y

    # -------------------------------------------------------------------------------- inference
    # Under tensor parallelism the output of every row-parallel projection is a partial sum;
    # the inference paths carry it as a "pending" value and reduce it together with the
    # residual add + RMSNorm that follows. With the symmetric-memory backend that is ONE fused
    # step: the row-parallel GEMM stores its tiles into the peers' staging over NVLink and the
    # reduce kernel does sum + residual + norm (dense layers), or the reduce kernel pushes a
    # MoE layer's combined output and does the same.
    def _tp_fused(self, rows: int) -> bool:
        return (self.tp is not None and self.tp.backend == "symm" and self.device.type == "cuda"
                and self.lora is None and rows <= self.tp.cap_rows)

    def _sw_pend(self, i: int, name: str, pend):
        """GLM-4 sandwich norm of a pending (inference) branch output: under TP the output is
        reduced first and returned as ("full", y) so that `_add_norm` does not reduce again."""
        if not self.cfg.sandwich_norm:
            return pend
        if isinstance(pend, tuple):
            pend = G.linear(pend[1], pend[2])
        if self.tp is not None:
            pend = self.tp.all_reduce(pend)
        y = rms_norm(pend, self.params[f"layers.{i}.{name}.weight"], self.cfg.rms_eps)
        return ("full", y) if self.tp is not None else y

    def _add_norm(self, pending, r, w):
        """(x, r') = add_rms_norm(allreduce(pending), r, w); pending is a tensor (partial or
        full output), ("gemm", a, W) meaning a @ W^T still to be computed, or ("full", y) an
        output already reduced over TP."""
        eps = self.cfg.rms_eps
        if isinstance(pending, tuple) and pending[0] == "full":
            y = pending[1]
            return (rms_norm(y, w, eps), y) if r is None else add_rms_norm(y, r, w, eps)
        if isinstance(pending, tuple):
            _, a, W = pending
            if self._tp_fused(a.shape[0]):
                return self.tp.symm().gemm_all_reduce(a, W, res=r, norm_w=w, eps=eps)
            pending = G.linear(a, W)
        if self.tp is not None:
            if self._tp_fused(pending.shape[0]):
                return self.tp.symm().all_reduce_add_norm(pending, r, w, eps)
            pending = self.tp.all_reduce(pending)
        if r is None:
            return rms_norm(pending, w, eps), pending
        return add_rms_norm(pending, r, w, eps)

    def _pending_out(self, a: torch.Tensor, name: str):
        """Row-parallel projection a @ W^T, deferred when it can fuse with its all-reduce."""
        if self._tp_fused(a.shape[0]):
            return ("gemm", a, self.params[name])
        return self._lin(a, name)

    def _pending_mlp(self, i: int, x: torch.Tensor):
        pre = f"layers.{i}.mlp."
        if i in self.router_cfgs or self.tp is None:
            return self._mlp_partial(i, x)
        return self._pending_out(self._lin_swiglu(x, pre + "gate_up_proj.weight"), pre + "down_proj.weight")

    @torch.no_grad()
    def forward_prefill(self, tokens: torch.Tensor, meta: VarlenMeta, cache: KVCache,
                        slots: torch.Tensor, record: list | None = None,
                        state_rows: torch.Tensor | None = None) -> torch.Tensor:
        """Packed prompt prefill. Writes K/V of every token to cache rows `slots` (int64 [T])
        (linear-attention layers: the final states of sequence b to row state_rows[b]).
        Returns the final hidden of every token [T, H]."""
        cfg = self.cfg
        self.sync_fp8()
        r = F.embedding(tokens.long(), self.params["embed_tokens.weight"])
        pend = None
        for i in range(cfg.num_layers):
            ln1 = self.params[f"layers.{i}.input_layernorm.weight"]
            x, r = (rms_norm(r, ln1, cfg.rms_eps), r) if pend is None else self._add_norm(pend, r, ln1)
            pre = f"layers.{i}.self_attn."
            post = self.params[f"layers.{i}.post_attention_layernorm.weight"]
            if self.gdn is not None and cfg.layer_is_linear(i):
                x2, r = self._add_norm(self._sw_pend(i, "post_self_attn_layernorm",
                                               self.gdn.attn(i, x, meta, cache, state_rows, pending=True)), r, post)
            elif self.gattn is not None:
                x2, r = self._add_norm(self._sw_pend(i, "post_self_attn_layernorm",
                                               self.gattn.attn(i, x, meta, cache, slots, pending=True)), r, post)
            elif self.mla is not None:
                x2, r = self._add_norm(self.mla.attn(i, x, meta, cache, slots, pending=True), r, post)
            else:
                qkv = self._lin(x, pre + "qkv_proj.weight")
                q, k, v = qk_norm_rope(qkv, self.params.get(pre + "q_norm.weight"),
                                       self.params.get(pre + "k_norm.weight"), meta.positions,
                                       self.rope_cos, self.rope_sin, self.nq, self.nkv,
                                       cfg.rms_eps, cfg.qk_norm)
                cache.k[i].index_copy_(0, slots, k)
                cache.v[i].index_copy_(0, slots, v)
                o = varlen_attention(q, k, v, meta)
                x2, r = self._add_norm(self._pending_out(o.reshape(x.shape[0], -1), pre + "o_proj.weight"),
                                       r, post)
            rec = record.append if (record is not None and i in self.router_cfgs) else None
            pend = self._mlp_partial(i, x2, record=rec) if rec is not None else self._pending_mlp(i, x2)
            pend = self._sw_pend(i, "post_mlp_layernorm", pend)
            if _dumper.enabled():
                _dumper.dump(f"layer{i:03d}_residual", r)
        y, _ = self._add_norm(pend, r, self.params["norm.weight"])
        if _dumper.enabled():
            _dumper.dump("final_hidden", y)
        return y

    @torch.no_grad()
    def forward_decode(self, tokens: torch.Tensor, positions: torch.Tensor, cache: KVCache,
                       page_table: torch.Tensor, ctx_lens: torch.Tensor, slots: torch.Tensor,
                       record: list | None = None, state_rows: torch.Tensor | None = None) -> torch.Tensor:
        """One token per sequence. tokens int [B]; positions int32 [B]; slots int64 [B]
        (cache row of the new token); ctx_lens int32 [B] = positions + 1. Returns hidden [B,H]."""
        cfg = self.cfg
        B = tokens.shape[0]
        self.sync_fp8()
        r = F.embedding(tokens.long(), self.params["embed_tokens.weight"])
        pend = None
        for i in range(cfg.num_layers):
            ln1 = self.params[f"layers.{i}.input_layernorm.weight"]
            x, r = (rms_norm(r, ln1, cfg.rms_eps), r) if pend is None else self._add_norm(pend, r, ln1)
            pre = f"layers.{i}.self_attn."
            post = self.params[f"layers.{i}.post_attention_layernorm.weight"]
            if self.gdn is not None and cfg.layer_is_linear(i):
                a = self.gdn.decode(i, x, cache, state_rows, pending=True)
            elif self.gattn is not None:
                a = self.gattn.decode(i, x, positions, cache, page_table, ctx_lens, slots, pending=True)
            elif self.mla is not None:
                a = self.mla.decode(i, x, positions, cache, page_table, ctx_lens, slots, pending=True)
            else:
                qkv = self._lin(x, pre + "qkv_proj.weight")
                q = qk_norm_rope_to_cache(qkv, self.params.get(pre + "q_norm.weight"),
                                          self.params.get(pre + "k_norm.weight"), positions,
                                          self.rope_cos, self.rope_sin, self.nq,
                                          self.nkv, cache.k[i], cache.v[i], slots,
                                          cfg.rms_eps, cfg.qk_norm)
                o = decode_attention(q, cache.k[i], cache.v[i], page_table, ctx_lens)
                a = self._pending_out(o.reshape(B, -1), pre + "o_proj.weight")
            x2, r = self._add_norm(self._sw_pend(i, "post_self_attn_layernorm", a), r, post)
            rec = None
            if record is not None and i in self.router_cfgs:
                # a [L_moe, B, k] buffer: the router writes layer i's routing straight into it
                rec = record[self.moe_index[i]] if isinstance(record, torch.Tensor) else record.append
            pend = self._mlp_partial(i, x2, record=rec) if rec is not None else self._pending_mlp(i, x2)
            pend = self._sw_pend(i, "post_mlp_layernorm", pend)
        y, _ = self._add_norm(pend, r, self.params["norm.weight"])
        return y

    @torch.no_grad()
    def mtp_infer(self, j: int, h: torch.Tensor, next_tokens: torch.Tensor, positions: torch.Tensor,
                  kc: torch.Tensor, vc: torch.Tensor, slots: torch.Tensor, meta: VarlenMeta | None = None,
                  page_table: torch.Tensor | None = None, ctx_lens: torch.Tensor | None = None):
        """Inference form of MTP layer j (the training form is in `mtp_loss`): row t combines the
        main model's final hidden h[t] (position t) with the embedding of token t + 1, runs layer
        j with its own paged K/V cache (kc / vc, rows `slots`), and returns (the layer output
        before the head norm, shared_head.norm of it) — the hidden whose LM-head distribution
        drafts token t + 2. With `meta` the rows are a packed prefill (varlen attention over the
        rows themselves); otherwise decode rows attending to the cache through `page_table` /
        `ctx_lens`. Standard softmax-attention layers only."""
        cfg = self.cfg
        p = f"layers.{j}."
        e = F.embedding(next_tokens.long(), self.params["embed_tokens.weight"])
        x = torch.cat([rms_norm(e, self.params[p + "enorm.weight"], cfg.rms_eps),
                       rms_norm(h.to(e.dtype), self.params[p + "hnorm.weight"], cfg.rms_eps)], -1)
        r = self._lin(x, p + "eh_proj.weight")
        xn = rms_norm(r, self.params[p + "input_layernorm.weight"], cfg.rms_eps)
        pre = p + "self_attn."
        qkv = self._lin(xn, pre + "qkv_proj.weight")
        T = xn.shape[0]
        if meta is not None:
            q, k, v = qk_norm_rope(qkv, self.params.get(pre + "q_norm.weight"),
                                   self.params.get(pre + "k_norm.weight"), positions,
                                   self.rope_cos, self.rope_sin, self.nq, self.nkv,
                                   cfg.rms_eps, cfg.qk_norm)
            kc.index_copy_(0, slots, k.to(kc.dtype))
            vc.index_copy_(0, slots, v.to(vc.dtype))
            o = varlen_attention(q, k, v, meta)
        else:
            q = qk_norm_rope_to_cache(qkv, self.params.get(pre + "q_norm.weight"),
                                      self.params.get(pre + "k_norm.weight"), positions,
                                      self.rope_cos, self.rope_sin, self.nq, self.nkv, kc, vc,
                                      slots, cfg.rms_eps, cfg.qk_norm)
            o = decode_attention(q, kc, vc, page_table, ctx_lens)
        x2, r = self._add_norm(self._pending_out(o.reshape(T, -1), pre + "o_proj.weight"), r,
                               self.params[p + "post_attention_layernorm.weight"])
        y, prev = self._add_norm(self._pending_mlp(j, x2), r, self.params[p + "shared_head.norm.weight"])
        return prev, y

    def flops_per_token(self, ctx: float) -> float:
        """Forward FLOPs per token (matmuls + attention at average context `ctx`)."""
        c = self.cfg
        attn = 4 * c.num_layers * c.num_heads * c.head_dim * ctx / 2  # causal: half the keys
        return 2 * c.active_params() + attn
