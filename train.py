"""Synchronous RL driver (colocated): one process per GPU.

    torchrun --nproc-per-node 8 train.py --model-name qwen3-30b-a3b --prompt-data data.jsonl \
        --rollout-batch-size 64 --n-samples-per-prompt 8 --rm-type math ...

Per rollout id: generate (this GPU's engine, this rank's prompt shard) -> release KV memory ->
train (log-probs, advantages, policy update, DP gradient reduction) -> periodic save ->
weight-version bump (colocated refit) -> periodic eval.

Reference: train.py:13-104 (the same loop across Ray actors and SGLang servers).
"""
from __future__ import annotations

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from miles_b200.checkpoint.torch_dist import (get_checkpoint_iteration, is_torch_dist,  # noqa: E402
                                              load_checkpoint, save_checkpoint, wait_async_save)
from miles_b200.orchestration.rollout_manager import RolloutManager  # noqa: E402
from miles_b200.orchestration.setup import (build_actor, build_critic, build_engine,  # noqa: E402
                                            build_engine_model, build_model, init_distributed,
                                            load_tokenizer)
from miles_b200.rollout.engine_client import LocalEngineClient  # noqa: E402
from miles_b200.trainer.train_actor import TrainActor  # noqa: E402
from miles_b200.trainer.lr_scheduler import restore_schedule, schedule_state  # noqa: E402
from miles_b200.utils.arguments import parse_args  # noqa: E402
from miles_b200.utils.misc import load_function, should_run_periodic_action  # noqa: E402
from miles_b200.utils.tracking import Tracker  # noqa: E402


def setup(args):
    ctx = init_distributed(args)
    if args.env_report:
        from miles_b200.utils.env_report import report

        report(ctx.rank)
    from miles_b200.utils import dumper

    dumper.configure(args, ctx.rank)
    model = build_model(args, ctx)
    actor = build_actor(args, model, ctx)
    engine_model = build_engine_model(args, model, ctx)
    overrides = None
    if getattr(args, "sglang_config", None):
        from miles_b200.rollout.sglang_config import load_deployment, overrides_for, pd_pairs

        engines, _ = load_deployment(args, list(range(ctx.world)))
        if pd_pairs(engines) is not None:
            raise ValueError("--sglang-config prefill / decode groups need disaggregated engines "
                             "(train_async.py); colocated engines run both phases")
        overrides = overrides_for(engines, ctx.rank)
    engine = build_engine(args, engine_model, ctx, overrides)
    tok = load_tokenizer(args)
    client = LocalEngineClient(engine, tok)
    ds_cls = load_function(args.data_source_path)
    data_source = ds_cls(args, tok)
    # prompts are sharded over data-parallel replicas: the ranks of one tensor-parallel group
    # generate (and train on) the same samples
    manager = RolloutManager(args, data_source, client, tok, ctx.dp_rank, ctx.dp_size)
    if args.use_session_server:
        # OpenAI-style session endpoint for agent rollouts (token-in / token-out trajectories)
        from miles_b200.rollout.session import launch_session_server

        manager.session_registry, _ = launch_session_server(args, tok, client)
    trainer = TrainActor(args, actor, ctx.dp_group, critic=build_critic(args, ctx),
                         data_parallel_size=ctx.dp_size)
    start = 0
    if args.load and is_torch_dist(args.load) and args.train_backend != "fsdp":
        actor._ensure_grads()
        info = load_checkpoint(args.load, model, actor.opt, load_optim=not args.no_load_optim)
        restore_schedule(actor, info)
        from miles_b200.utils.ci_utils import check_model_hashes

        check_model_hashes(args, model, info["iteration"], ctx.rank)
        start = info.get("extra", {}).get("rollout_id", info["iteration"]) + 1
        data_source.load(start - 1)
    if args.start_rollout_id is not None:
        start = args.start_rollout_id
    trainer.init_ref()
    tracker = Tracker(args, ctx.rank)
    from miles_b200.orchestration.fault_tolerance import EngineSupervisor, default_store

    manager.supervisor = EngineSupervisor(args, engine, lambda: build_engine(args, engine_model, ctx, overrides),
                                          client, ctx.rank, ctx.world, default_store())
    return ctx, model, actor, engine, manager, trainer, tracker, start, data_source


def train(args):
    ctx, model, actor, engine, manager, trainer, tracker, start, data_source = setup(args)
    from miles_b200.utils.profile_utils import TrainProfiler

    profiler = TrainProfiler(args, ctx.rank)
    num_rollout = args.num_rollout
    if args.eval_interval and not args.skip_eval_before_train:
        tracker.log(manager.eval(start), start)
    for rollout_id in range(start, num_rollout):
        actor.release_grads()
        reload_groups = args.offload_train and dist.is_initialized() and dist.get_world_size() > 1
        if reload_groups:
            # the trainer's DP / CP / pipeline communicators are idle during the rollout: free
            # their device buffers and rebuild them (rebinding every holder) before training
            from miles_b200.parallel import pp as _pp
            from miles_b200.parallel.reloadable import REGISTRY

            REGISTRY.destroy()
        engine = manager.supervisor.before_rollout(rollout_id)  # recovers a dead engine
        data = manager.generate(rollout_id)
        manager.supervisor.after_rollout()
        engine.release_memory(args.offload_rollout_level)
        if reload_groups:
            REGISTRY.reload([ctx, model, actor, trainer, _pp._TIED_GROUPS])
        if args.debug_rollout_only:
            tracker.log(data["metrics"], rollout_id)
            continue
        profiler.start("train_overall")
        m = trainer.train(rollout_id, data)
        trainer.after_update(rollout_id)
        if args.train_backend == "fsdp":  # HF policy under FSDP2 -> the engine's Transformer
            from miles_b200.checkpoint.hf import load_hf_tensors

            load_hf_tensors(model, actor.export_hf_state())
            model.weight_version += 1
        if engine.model is not model:  # pipeline stages -> the engine's full-depth copy
            from miles_b200.parallel.pp import gather_full_weights

            gather_full_weights(model, engine.model)
        profiler.stop("train_overall")
        profiler.step()
        m.update(data["metrics"])
        if (should_run_periodic_action(rollout_id, args.save_interval, num_rollout) and args.save
                and args.train_backend != "fsdp"):
            save_checkpoint(args.save, rollout_id, model, actor.opt, extra={"rollout_id": rollout_id, **schedule_state(actor)},
                            save_optim=not args.no_save_optim, async_save=args.async_save)
            data_source.save(rollout_id)
            if args.critic_save and trainer.critic is not None:
                # the PPO critic: body in torch_dist layout plus its value head
                cr = trainer.critic
                save_checkpoint(args.critic_save, rollout_id, cr.model, cr.body.opt,
                                extra={"rollout_id": rollout_id}, save_optim=not args.no_save_optim)
                torch.save(cr.head.detach().cpu(), os.path.join(
                    args.critic_save, f"iter_{rollout_id:07d}", "value_head.pt"))
            from miles_b200.utils.ci_utils import save_model_hashes

            save_model_hashes(args, model, rollout_id, ctx.rank)
            if args.save_hf:
                from miles_b200.checkpoint.hf import save_hf

                # the TP group of replica 0 (save_hf gathers over it); under EP the ranks that
                # hold one copy of every expert too (the first tp * ep ranks with TP-split
                # experts, the first max(tp, ep) with whole experts)
                if model.ep is None:
                    saver = ctx.dp_rank == 0
                else:
                    tp_n, ep_n = model.tp_size, model.ep.size
                    saver = ctx.rank < (tp_n * ep_n if model.expert_tp > 1 else max(tp_n, ep_n))
                if saver:
                    save_hf(model, args.save_hf.format(rollout_id=rollout_id))
        # colocated refit: the engine reads the trainer's parameter buffer in place
        m["rollout/weight_version"] = model.weight_version
        if manager.supervisor.enabled:
            m["fault_tolerance/recoveries"] = manager.supervisor.recoveries
        if should_run_periodic_action(rollout_id, args.eval_interval, num_rollout):
            m.update(manager.eval(rollout_id))
        tracker.log(m, rollout_id)
    wait_async_save()
    manager.supervisor.close()
    if args.ci_metric_checker_key:
        from miles_b200.utils.metric_checker import check_metric

        check_metric(args, tracker.history)
    tracker.finish()
    return tracker.history


if __name__ == "__main__":
    train(parse_args())
