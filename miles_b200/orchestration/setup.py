"""Process-level setup shared by train.py / train_async.py: distributed init, model, engine,
actor, tokenizer and the rollout manager for this GPU process.

Reference: miles/ray/placement_group.py (create_*), miles/ray/train_actor.py (init:
env ranks, init_process_group(nccl) + gloo group :30-104), megatron_utils/actor.py init
(:52-194: model, optimizer, checkpoint load, ref backup, weight updater).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from miles_b200.engine.engine import RolloutEngine
from miles_b200.models.config import ModelConfig, preset
from miles_b200.models.transformer import Transformer
from miles_b200.ops.rl import PolicyLossCfg
from miles_b200.parallel.reloadable import REGISTRY as _RG
from miles_b200.trainer.actor import Actor, ActorConfig
from miles_b200.trainer.lr_scheduler import schedule_from_args
from miles_b200.utils.misc import load_function


@dataclass
class ProcessContext:
    rank: int
    world: int
    local_rank: int
    device: torch.device
    dp_group: object = None
    gloo_group: object = None
    tp_group: object = None        # tensor-parallel group (consecutive ranks)
    ep_group: object = None        # expert-parallel group (consecutive ranks)
    expert_dp_group: object = None  # ranks holding the same experts
    cp_group: object = None        # context-parallel group (consecutive ranks)
    pp_group: object = None        # pipeline group (one rank per stage)
    dp_rank: int = 0
    dp_size: int = 1


def _groups(world: int, size: int):
    """(consecutive groups of `size`, strided groups across them) as rank lists."""
    blocks = [list(range(b, b + size)) for b in range(0, world, size)]
    strided = [list(range(i, world, size)) for i in range(size)]
    return blocks, strided


def init_distributed(args) -> ProcessContext:
    if getattr(args, "http_proxy", None):  # proxy for the HTTP clients (reward models, routers)
        os.environ.setdefault("http_proxy", args.http_proxy)
        os.environ.setdefault("https_proxy", args.http_proxy)
    # --train-env-vars: JSON object of environment variables for the training process
    env = getattr(args, "train_env_vars", None)
    if env and env != "{}":
        os.environ.update({k: str(v) for k, v in json.loads(env).items()})
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and not os.environ.get("MILES_B200_FORCE_CPU")
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    dp = gloo = None
    if world > 1 and not dist.is_initialized():
        import datetime

        backend = "nccl" if use_cuda else "gloo"
        kw = {"device_id": dev} if use_cuda else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(minutes=args.distributed_timeout_minutes), **kw)
    ctx = ProcessContext(rank, world, local, dev)
    if world > 1:
        dp = dist.group.WORLD
        gloo = _RG.new_group(backend="gloo", tag="keep") if use_cuda else dp
        ctx.dp_group, ctx.gloo_group, ctx.dp_rank, ctx.dp_size = dp, gloo, rank, world
        tp = getattr(args, "tensor_model_parallel_size", 1)
        ep = getattr(args, "expert_model_parallel_size", 1)
        cp = getattr(args, "context_parallel_size", 1)
        pp = getattr(args, "pipeline_model_parallel_size", 1)
        if pp > 1:
            if tp > 1 or ep > 1 or cp > 1:
                raise ValueError("pipeline parallelism is supported with data parallelism only")
            from miles_b200.parallel.pp import register_tied_embedding_groups

            # stage s holds ranks [s*D, (s+1)*D) (its DP group); pipeline d is {d + s*D}
            D = world // pp
            for d in range(D):
                g = _RG.new_group([d + s_ * D for s_ in range(pp)])
                if rank % D == d:
                    ctx.pp_group = g
            for s_ in range(pp):
                ranks = list(range(s_ * D, (s_ + 1) * D))
                g = _RG.new_group(ranks)
                if rank in ranks:
                    ctx.dp_group = g
            register_tied_embedding_groups(world, pp)
            ctx.dp_rank, ctx.dp_size = rank % D, D
        if cp > 1 and ep > 1:
            raise ValueError("context parallelism combined with expert parallelism is not supported")
        if cp > 1 and tp > 1:
            # TP x CP (rank = replica * tp * cp + c * tp + t): a CP group is the ranks with the
            # same TP rank in one replica; gradients reduce over all ranks of the same TP rank
            # (the TP block below), data is sharded over replicas of tp * cp ranks
            blk = tp * cp
            for b in range(0, world, blk):
                for t in range(tp):
                    ranks = [b + c * tp + t for c in range(cp)]
                    g = _RG.new_group(ranks)
                    if rank in ranks:
                        ctx.cp_group = g
        elif cp > 1:
            # CP groups are consecutive ranks; gradients reduce over every rank (DP x CP),
            # data is sharded over DP replicas only
            blocks, _ = _groups(world, cp)
            for ranks in blocks:
                g = _RG.new_group(ranks)
                if rank in ranks:
                    ctx.cp_group = g
            ctx.dp_rank, ctx.dp_size = rank // cp, world // cp
        if tp > 1:
            # TP groups are consecutive ranks (one NVSwitch domain); DP across them
            blocks, strided = _groups(world, tp)
            for ranks in blocks:
                g = _RG.new_group(ranks, tag="rollout")
                if rank in ranks:
                    ctx.tp_group = g
            for ranks in strided:
                g = _RG.new_group(ranks)
                if rank in ranks:
                    ctx.dp_group = g
            ctx.dp_rank, ctx.dp_size = rank // tp, world // tp
            if cp > 1:
                ctx.dp_rank, ctx.dp_size = rank // (tp * cp), world // (tp * cp)
        etp = getattr(args, "expert_tensor_parallel_size", None)
        if ep > 1 and tp > 1 and etp == 1 and ep % tp and tp % ep:
            raise ValueError(f"whole experts under TP need EP ({ep}) and TP ({tp}) to divide one another")
        if ep > 1 and tp > 1 and etp != 1:
            # TP x EP: attention heads and every expert's FFN width split over the TP group
            # (expert-tensor parallel = TP); experts split over EP groups of the ranks with the
            # same TP rank (consecutive data-parallel replicas); expert gradients reduce over
            # the replicas of the same (TP rank, EP rank)
            D = world // tp
            if D % ep:
                raise ValueError(f"{D} data-parallel replicas do not split into EP groups of {ep}")
            for t in range(tp):
                for b in range(0, D, ep):
                    ranks = [t + tp * (b + e) for e in range(ep)]
                    g = _RG.new_group(ranks, tag="rollout")
                    if rank in ranks:
                        ctx.ep_group = g
                for e in range(ep):
                    ranks = [t + tp * (b + e) for b in range(0, D, ep)]
                    g = _RG.new_group(ranks)
                    if rank in ranks:
                        ctx.expert_dp_group = g
        elif ep > 1:
            # EP alone, or with whole experts under TP: EP groups of consecutive ranks
            blocks, strided = _groups(world, ep)
            for ranks in blocks:
                g = _RG.new_group(ranks, tag="rollout")
                if rank in ranks:
                    ctx.ep_group = g
            for ranks in strided:
                g = _RG.new_group(ranks)
                if rank in ranks:
                    ctx.expert_dp_group = g
    return ctx


def model_config(args) -> ModelConfig:
    if args.model_name:
        cfg = preset(args.model_name)
    elif args.hf_checkpoint:
        cfg = ModelConfig.from_hf(args.hf_checkpoint)
    else:
        raise ValueError("pass --model-name <preset> or --hf-checkpoint <dir>")
    if getattr(args, "enable_mtp_training", False):
        import dataclasses

        depth = (getattr(args, "mtp_num_layers", None) or cfg.extra.get("num_nextn_predict_layers")
                 or 1)
        cfg = dataclasses.replace(cfg, mtp_num_layers=depth)
    return cfg


def load_tokenizer(args):
    if not args.hf_checkpoint or not os.path.isdir(args.hf_checkpoint):
        return None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(args.hf_checkpoint, trust_remote_code=True)
    except Exception:
        return None
    if getattr(args, "chat_template_path", None):
        # --chat-template-path: a Jinja chat template file replacing the tokenizer's own
        with open(args.chat_template_path) as f:
            tok.chat_template = f.read()
    return tok


def build_model(args, ctx: ProcessContext) -> Transformer:
    if getattr(args, "custom_megatron_init_path", None):
        # user initialisation after the process groups exist (reference initialize.py:106-110)
        load_function(args.custom_megatron_init_path)(args)
    cfg = model_config(args)
    dtype = torch.bfloat16 if ctx.device.type == "cuda" else torch.float32
    provider = None
    if getattr(args, "custom_model_provider_path", None):
        # custom model provider: fn(args, cfg) returning a ModelConfig to build, or a built
        # Transformer (the role of the reference's Megatron model_provider hook)
        provider = load_function(args.custom_model_provider_path)(args, cfg)
        if isinstance(provider, ModelConfig):
            cfg, provider = provider, None
    model = provider if provider is not None else Transformer(
                        cfg, device=ctx.device, dtype=dtype, seed=args.seed, tp_group=ctx.tp_group,
                        ep_group=ctx.ep_group, cp_group=ctx.cp_group, pp_group=ctx.pp_group,
                        vpp=getattr(args, "virtual_pipeline_model_parallel_size", None) or 1,
                        pp_first_layers=getattr(args, "decoder_first_pipeline_num_layers", None),
                        pp_last_layers=getattr(args, "decoder_last_pipeline_num_layers", None),
                        etp=getattr(args, "expert_tensor_parallel_size", None),
                        tp_cap_rows=max(4096, getattr(args, "max_tokens_per_gpu", 0) or 0))
    model.mtp_train = bool(getattr(args, "enable_mtp_training", False))
    # activation recompute (Megatron flags): granularity "full" recomputes whole layers; method
    # "block" limits it to the first --recompute-num-layers layers of this rank ("uniform"
    # recomputes every layer, one checkpoint per layer); granularity "none" stores activations
    gran = getattr(args, "recompute_granularity", "full") or "none"
    if gran not in ("full", "selective", "none"):
        raise ValueError(f"unknown --recompute-granularity {gran}")
    model.recompute = gran != "none"
    if gran != "none" and getattr(args, "recompute_method", "uniform") == "block":
        model.recompute_layers = int(args.recompute_num_layers)
    if getattr(args, "sequence_parallel", False) and model.tp is not None:
        model.sequence_parallel = True
    if getattr(args, "vocab_parallel_logprob", False) and model.tp is not None:
        model.vocab_parallel_logprob = True
    loaded = False
    if args.load:
        from miles_b200.checkpoint.torch_dist import is_torch_dist

        if is_torch_dist(args.load):
            loaded = True  # the actor loads it (with optimizer state) once built
    if not loaded and args.hf_checkpoint and os.path.isdir(args.hf_checkpoint) and any(
            f.endswith(".safetensors") for f in os.listdir(args.hf_checkpoint)):
        from miles_b200.checkpoint.hf import load_hf

        load_hf(model, args.hf_checkpoint)
    fmt, recipe = getattr(args, "fp8_format", None), getattr(args, "fp8_recipe", "blockwise")
    if fmt:
        # unified block-scaled fp8 training + rollout (the reference's --fp8-format e4m3
        # --fp8-recipe blockwise with fp8 rollout engines)
        if fmt != "e4m3" or recipe != "blockwise":
            raise ValueError(f"fp8 supports --fp8-format e4m3 --fp8-recipe blockwise (got {fmt} / {recipe})")
        model.enable_fp8()
    if os.environ.get("OPEN_TRAINING_INT4_FAKE_QAT_FLAG", "0") == "1":
        # int4 quantisation-aware training of the routed experts (the reference's switch)
        model.enable_int4_qat(int(os.environ.get("OPEN_TRAINING_INT4_GROUP_SIZE", "128")))
    if getattr(args, "lora_rank", 0):
        from miles_b200.models.lora import LoRA

        model.lora = LoRA(model, args.lora_rank, args.lora_alpha, args.target_modules,
                          args.lora_dropout, seed=args.seed, exclude=args.exclude_modules)
        if args.lora_adapter_path:
            model.lora.load(args.lora_adapter_path)
    return model


def build_actor(args, model: Transformer, ctx: ProcessContext) -> Actor:
    from miles_b200.trainer.is_functions import KERNEL_MODES

    tis_path = args.custom_tis_function_path
    tis_mode = KERNEL_MODES.get(tis_path or "", "tis")
    loss = PolicyLossCfg(eps_clip=args.eps_clip, eps_clip_high=args.eps_clip_high,
                         eps_clip_c=args.eps_clip_c, use_tis=args.use_tis,
                         tis_clip_low=args.tis_clip_low, tis_clip=args.tis_clip,
                         tis_mode=tis_mode,
                         custom_tis_path=None if tis_path in KERNEL_MODES or not tis_path else tis_path,
                         loss_type=args.loss_type, custom_loss_path=args.custom_loss_function_path,
                         unbiased_kl=args.use_unbiased_kl,
                         custom_pg_loss_reducer_path=args.custom_pg_loss_reducer_function_path,
                         use_opsm=args.use_opsm, opsm_delta=args.opsm_delta,
                         gspo=args.advantage_estimator == "gspo",
                         kl_coef=args.kl_loss_coef if args.use_kl_loss else 0.0,
                         kl_type=args.kl_loss_type if args.use_kl_loss else "none")
    placement = "host" if args.optimizer_cpu_offload else "auto"
    cfg = ActorConfig(lr=args.lr, betas=(args.adam_beta1, args.adam_beta2),
                      weight_decay=args.weight_decay, clip_grad=args.clip_grad,
                      max_tokens_per_gpu=args.max_tokens_per_gpu or 16384, loss=loss,
                      entropy_coef=args.entropy_coef, per_token_loss=args.calculate_per_token_loss,
                      temperature=args.rollout_temperature,
                      use_rollout_logprobs=args.use_rollout_logprobs,
                      use_routing_replay=args.use_routing_replay,
                      grad_dtype=torch.float32 if (ctx.device.type != "cuda" or args.accumulate_allreduce_grads_in_fp32) else torch.bfloat16,
                      optimizer_placement=placement,
                      logprob_chunk=args.log_probs_chunk_size if args.log_probs_chunk_size > 0 else 4096,
                      mtp_loss_scale=(args.mtp_loss_scaling_factor
                                      if getattr(args, "enable_mtp_training", False) else 0.0),
                      adam_eps=args.adam_eps, lr_schedule=schedule_from_args(args), tis_args=args,
                      micro_batching="balanced" if args.use_dynamic_batch_size else "fixed",
                      micro_batch_size=args.micro_batch_size,
                      log_probs_max_tokens_per_gpu=args.log_probs_max_tokens_per_gpu,
                      memory_margin_bytes=args.train_memory_margin_bytes,
                      old_logp_from_forward=_old_logp_from_forward(args),
                      grad_reduce=getattr(args, "grad_reduce", "nccl"),
                      offload_optimizer=bool(getattr(args, "offload_train", False)
                                             and getattr(args, "colocate", False)))
    if getattr(args, "train_backend", "b200") == "fsdp":
        # HF model under FSDP2 (trainer/fsdp_actor.py); `model` is then the engine's Transformer,
        # refreshed from the gathered HF state after every step
        from miles_b200.checkpoint.hf import load_hf_tensors
        from miles_b200.trainer.fsdp_actor import FSDPActor

        if args.use_kl_loss or args.kl_coef or args.use_routing_replay:
            raise ValueError("--train-backend fsdp supports no reference-model KL and no routing replay")
        if not args.hf_checkpoint:
            raise ValueError("--train-backend fsdp loads the policy from --hf-checkpoint")
        actor = FSDPActor(args.hf_checkpoint, cfg, dp_group=ctx.dp_group, device=ctx.device,
                          dtype=model.dtype)
        load_hf_tensors(model, actor.export_hf_state())
        actor.engine_model = model
        return actor
    actor = Actor(model, cfg, dp_group=ctx.dp_group)
    actor.expert_dp_group = ctx.expert_dp_group
    return actor


def _old_logp_from_forward(args) -> bool:
    """Take the old log-probs from the training forward instead of a separate pass when nothing
    needs them before the update: one optimizer step per rollout, an estimator that does not
    use them (GRPO / GSPO), no KL-shaped rewards, no old-actor weights, no mismatch report. The
    values are bitwise those of the separate pass (same weights, batch-invariant kernels)."""
    return (getattr(args, "num_steps_per_rollout", None) in (None, 1)
            and args.advantage_estimator in ("grpo", "gspo") and not args.kl_coef
            and not getattr(args, "keep_old_actor", False)
            and not getattr(args, "get_mismatch_metrics", False)
            and getattr(args, "train_backend", "b200") != "fsdp")


def sglang_engine_kwargs(sg: dict) -> dict:
    """RolloutEngine arguments from the forwarded `--sglang-*` flags that have a counterpart in
    this engine (SGLang server argument names): mem_fraction_static -> KV pool share,
    max_running_requests -> batch slots, chunked_prefill_size -> packed-prefill token budget,
    disable_cuda_graph -> no decode graphs, context_length -> longest sequence,
    num_continuous_decode_steps -> decode steps per host visit, speculative_algorithm
    (NEXTN / EAGLE / MTP) -> speculative rollout with the MTP draft. Other SGLang flags (kernels,
    schedulers and servers this engine does not have) are accepted and ignored."""

    def flag(v):
        return v in (True, "true", "True", "1", 1, None, "")

    out = {}
    if "mem_fraction_static" in sg:
        out["mem_fraction"] = float(sg["mem_fraction_static"])
    if "max_running_requests" in sg:
        out["max_batch"] = int(sg["max_running_requests"])
    if "chunked_prefill_size" in sg and int(sg["chunked_prefill_size"]) > 0:
        out["prefill_tokens"] = int(sg["chunked_prefill_size"])
    if "disable_cuda_graph" in sg and flag(sg["disable_cuda_graph"]):
        out["use_cuda_graph"] = False
    if "context_length" in sg:
        out["context_length"] = int(sg["context_length"])
    if "num_continuous_decode_steps" in sg:
        out["steps_per_sync"] = int(sg["num_continuous_decode_steps"])
    if sg.get("speculative_algorithm"):
        out["speculative"] = str(sg["speculative_algorithm"]).lower()
    return out


def build_engine(args, model: Transformer, ctx: ProcessContext,
                 overrides: dict | None = None) -> RolloutEngine:
    """The rank's rollout engine; `overrides`: SGLang flags of its `--sglang-config` group,
    applied over the forwarded `--sglang-*` ones."""
    sg = sglang_engine_kwargs({**(getattr(args, "sglang_args", {}) or {}), **(overrides or {})})
    max_len = (args.rollout_max_prompt_len or 1024) + (args.rollout_max_response_len or 1024)
    if args.rollout_max_context_len:
        max_len = max(max_len, args.rollout_max_context_len)
    max_len = max(max_len, sg.pop("context_length", 0))
    kw = dict(max_batch=args.rollout_max_batch, mem_fraction=0.85,
              use_cuda_graph=not args.no_cuda_graph)
    kw.update(sg)
    return RolloutEngine(model, num_pages=None if ctx.device.type == "cuda" else 4096,
                         max_pages_per_seq=(max_len + 63) // 64 + 1, **kw)


def build_critic(args, ctx: ProcessContext):
    """PPO value model (same architecture, its own weights and optimizer) when
    --advantage-estimator ppo; None otherwise."""
    if not getattr(args, "use_critic", False):
        return None
    from miles_b200.trainer.critic import Critic

    cfg = model_config(args)
    dtype = torch.bfloat16 if ctx.device.type == "cuda" else torch.float32
    body = Transformer(cfg, device=ctx.device, dtype=dtype, seed=args.seed + 1)
    if args.critic_load:
        from miles_b200.checkpoint.torch_dist import is_torch_dist, load_checkpoint

        if is_torch_dist(args.critic_load):
            load_checkpoint(args.critic_load, body)
    acfg = ActorConfig(lr=args.critic_lr, betas=(args.adam_beta1, args.adam_beta2),
                       adam_eps=args.adam_eps,
                       lr_schedule=schedule_from_args(args, lr=args.critic_lr,
                                                      warmup_iters=args.critic_lr_warmup_iters),
                       weight_decay=args.weight_decay, clip_grad=args.clip_grad,
                       max_tokens_per_gpu=args.max_tokens_per_gpu or 16384,
                       grad_dtype=torch.float32 if ctx.device.type != "cuda" else torch.bfloat16,
                       optimizer_placement="host" if args.optimizer_cpu_offload else "auto",
                       micro_batching="balanced" if args.use_dynamic_batch_size else "fixed",
                       micro_batch_size=args.micro_batch_size)
    critic = Critic(body, acfg, value_clip=args.value_clip, dp_group=ctx.dp_group)
    if args.critic_load:
        from miles_b200.checkpoint.torch_dist import get_checkpoint_iteration

        it = get_checkpoint_iteration(args.critic_load)
        head = os.path.join(args.critic_load, f"iter_{it:07d}", "value_head.pt") if it is not None else ""
        if head and os.path.exists(head):
            with torch.no_grad():
                critic.head.copy_(torch.load(head, weights_only=True).to(critic.head.device))
    return critic


def build_engine_model(args, model: Transformer, ctx: ProcessContext) -> Transformer:
    """The model the colocated rollout engine runs. Pipeline stages hold a slice of the layers,
    so under pipeline parallelism every rank also keeps a full-depth copy that is refreshed from
    the stages after each training step (parallel/pp.py gather_full_weights)."""
    if model.pp is None:
        return model
    from miles_b200.parallel.pp import gather_full_weights

    full = Transformer(model.cfg, device=ctx.device, dtype=model.dtype, materialize=False)
    gather_full_weights(model, full)
    return full
