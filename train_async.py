"""Asynchronous RL driver with disaggregated rollout: trainer GPUs and rollout GPUs are separate
processes of one torchrun world, and generation of the next batch overlaps training.

    torchrun --nproc-per-node 8 train_async.py --actor-num-gpus-per-node 4 \
        --rollout-num-gpus 4 --model-name ... --prompt-data ... [--fully-async] \
        [--update-weights-interval 1] [--update-weight-quant fp8] [--partial-rollout]

Ranks [0, T) train (T = actor nodes x GPUs per node; data parallel over them, sharded
optimizer); ranks [T, T + R) each run a rollout engine over their shard of the prompt stream.

One-step-ahead pipeline (default), the reference's schedule:
    engines : gen(0) send | gen(1) send | refit(0) gen(2) send | refit(1) gen(3) ...
    trainers: recv(0) | train(0) recv(1) refit(0) | train(1) recv(2) refit(1) | ...
  gen(r) therefore runs while train(r-1) does, under the weights of train(r-2). A refit after
  train(j) happens when (j + 1) % --update-weights-interval == 0 and an engine batch will use
  it; it is a bucketed NCCL broadcast of the flat parameter buffer from trainer rank 0
  (miles_b200/parallel/refit.py), optionally fp8 block-quantised.

--fully-async: each engine rank runs a background worker (miles_b200/rollout/fully_async.py)
that keeps groups in flight continuously; a refit pauses it (aborting in-flight requests,
recycling partial samples with --partial-rollout) and batches older than
--max-weight-staleness weight versions are dropped.

Reference: train_async.py:12-73 (prefetch generate(rollout_id + 1) while training rollout_id,
refit every --update-weights-interval after draining the pending generate, colocation
forbidden) and examples/fully_async.
"""
from __future__ import annotations

import datetime
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from miles_b200.orchestration.rollout_manager import RolloutManager  # noqa: E402
from miles_b200.orchestration.setup import (ProcessContext, build_actor, build_engine,  # noqa: E402
                                            build_model, load_tokenizer)
from miles_b200.parallel.refit import make_refit  # noqa: E402
from miles_b200.rollout.engine_client import LocalEngineClient  # noqa: E402
from miles_b200.trainer.train_actor import TrainActor  # noqa: E402
from miles_b200.trainer.lr_scheduler import restore_schedule, schedule_state  # noqa: E402
from miles_b200.utils.arguments import parse_args  # noqa: E402
from miles_b200.utils.misc import load_function, should_run_periodic_action  # noqa: E402
from miles_b200.utils.tracking import Tracker  # noqa: E402


def _init(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    T = args.actor_num_nodes * args.actor_num_gpus_per_node
    R = args.rollout_num_gpus
    if args.colocate:
        raise ValueError("train_async.py runs disaggregated: --colocate is not supported")
    if world != T + R or R < 1 or T < 1:
        raise ValueError(f"world size {world} must equal trainer GPUs ({T}) + rollout GPUs ({R})")
    use_cuda = torch.cuda.is_available() and not os.environ.get("MILES_B200_FORCE_CPU")
    if use_cuda:
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    if not dist.is_initialized():
        kw = {"device_id": dev} if use_cuda else {}
        dist.init_process_group("nccl" if use_cuda else "gloo",
                                timeout=datetime.timedelta(minutes=args.distributed_timeout_minutes), **kw)
    train_ranks = list(range(T))
    engine_ranks = list(range(T, T + R))
    # every rank creates every group (new_group is collective)
    train_group = dist.new_group(train_ranks)
    train_gloo = dist.new_group(train_ranks, backend="gloo")
    refit_group = dist.new_group([0] + engine_ranks)
    data_gloo = dist.new_group([0] + engine_ranks, backend="gloo")
    ctx = ProcessContext(rank, world, local, dev, train_group if rank < T else None,
                         train_gloo if rank < T else None)
    return ctx, T, R, train_group, train_gloo, refit_group, data_gloo


def _merge(parts: list[dict]) -> dict:
    parts = [p for p in parts if p is not None]  # prefill ranks contribute no samples
    out: dict = {}
    for p in parts:
        for k, v in p.items():
            if k == "metrics":
                continue
            out.setdefault(k, []).extend(v)
    ms = [p.get("metrics", {}) for p in parts]
    out["metrics"] = {k: sum(m.get(k, 0.0) for m in ms) / len(ms) for k in ms[0]} if ms else {}
    return out


def _split(data: dict, n: int, i: int) -> dict:
    """Trainer i's share: contiguous slices of whole prompt groups."""
    N = len(data["tokens"])
    per = N // n
    sl = slice(i * per, (i + 1) * per if i < n - 1 else N)
    return {k: (v[sl] if isinstance(v, list) else v) for k, v in data.items()}


def _refit_due(j: int, args, num_rollout: int, start: int) -> bool:
    """A refit follows train(j) when the interval says so and gen(j + 2) will use it."""
    return j >= start and (j + 1) % args.update_weights_interval == 0 and j + 2 < num_rollout


def run_trainer(args, ctx, T, train_gloo, refit_group, data_gloo):
    model = build_model(args, ctx)
    actor = build_actor(args, model, ctx)
    trainer = TrainActor(args, actor, ctx.dp_group)
    trainer.init_ref()
    # only trainer rank 0 belongs to the refit group (it holds the full parameters)
    refit = make_refit(model, refit_group, src=0, bucket_bytes=args.update_weight_buffer_size,
                       mode="fp8" if args.update_weight_quant == "fp8" else "bf16",
                       transport=args.update_weight_transport) if ctx.rank == 0 else None
    tracker = Tracker(args, ctx.rank)
    start, N = 0, args.num_rollout
    if ctx.rank == 0:
        refit.sync()  # initial weights to the engines

    def recv():
        mine = [None]
        if ctx.rank == 0:
            parts = [None] * dist.get_world_size(data_gloo)
            dist.gather_object(None, parts, dst=0, group=data_gloo)
            data = _merge([p for p in parts[1:]])
            shards = [_split(data, T, i) for i in range(T)]
        else:
            shards = None
        if T > 1:
            dist.scatter_object_list(mine, shards, src=0, group=train_gloo)
            return mine[0]
        return shards[0]

    data = recv()
    for j in range(start, N):
        m = trainer.train(j, data)
        trainer.after_update(j)
        m.update(data.get("metrics", {}))
        if j + 1 < N:
            data = recv()
        if _refit_due(j, args, N, start):
            if ctx.rank == 0:
                m.update(refit.sync())
                if args.check_weight_update_equal:
                    from miles_b200.parallel.refit import verify_weights_equal

                    m.update(verify_weights_equal(model, refit_group, 0, args.update_weight_quant != "fp8"))
        m["rollout/weight_version"] = model.weight_version
        if should_run_periodic_action(j, args.save_interval, N) and args.save:
            from miles_b200.checkpoint.torch_dist import save_checkpoint

            save_checkpoint(args.save, j, model, actor.opt, extra={"rollout_id": j, **schedule_state(actor)},
                            save_optim=not args.no_save_optim, process_group=ctx.dp_group)
        tracker.log(m, j)
    tracker.finish()
    return tracker.history


def _pd_roles(args, T: int, R: int):
    """Prefill / decode disaggregation (--prefill-num-servers K): the first K engine ranks
    prefill, the other R - K decode; decode rank j is paired with prefill rank j (K = R - K).
    Returns (prefill ranks, decode ranks) or None."""
    K = getattr(args, "prefill_num_servers", None) or 0
    if getattr(args, "sglang_config", None):
        from miles_b200.rollout.sglang_config import load_deployment, pd_pairs

        if K:
            raise ValueError("--sglang-config and --prefill-num-servers are exclusive")
        roles = pd_pairs(load_deployment(args, list(range(T, T + R)))[0])
        if roles is not None and args.fully_async:
            raise ValueError("prefill / decode groups are not supported with --fully-async")
        return roles
    if not K:
        return None
    if 2 * K != R:
        raise ValueError(f"--prefill-num-servers {K}: pairs one prefill rank with one decode rank, "
                         f"so it must be half of the {R} rollout GPUs")
    if args.fully_async:
        raise ValueError("--prefill-num-servers is not supported with --fully-async")
    eng = list(range(T, T + R))
    return eng[:K], eng[K:]


def _overrides(args, ctx, T: int, R: int) -> dict | None:
    """SGLang-flag overrides of this rank's `--sglang-config` engine group."""
    if not getattr(args, "sglang_config", None):
        return None
    from miles_b200.rollout.sglang_config import load_deployment, overrides_for

    return overrides_for(load_deployment(args, list(range(T, T + R)))[0], ctx.rank)


def run_prefill(args, ctx, T, R, refit_group, data_gloo, pre: list[int], dec: list[int]):
    """A prefill rank: per rollout step, prefill the requests of its paired decode rank until it
    ends the step; take part in the refits like every engine rank; contribute no samples."""
    from miles_b200.rollout.pd import serve_prefill_step

    model = build_model(args, ctx)
    engine = build_engine(args, model, ctx, _overrides(args, ctx, T, R))
    peer = dec[pre.index(ctx.rank)]
    refit = make_refit(model, refit_group, src=0, bucket_bytes=args.update_weight_buffer_size,
                       mode="fp8" if args.update_weight_quant == "fp8" else "bf16",
                       transport=args.update_weight_transport)
    refit.sync()
    start, N = 0, args.num_rollout
    for r in range(start, N):
        if r >= start + 2 and _refit_due(r - 2, args, N, start):
            refit.sync()
            if args.check_weight_update_equal:
                from miles_b200.parallel.refit import verify_weights_equal

                verify_weights_equal(model, refit_group, 0, args.update_weight_quant != "fp8")
        n = serve_prefill_step(engine, peer)
        print(f"[prefill rank {ctx.rank}] rollout {r}: prefilled {n} requests for rank {peer}", flush=True)
        engine.release_memory()
        dist.gather_object(None, None, dst=0, group=data_gloo)
    return []


def run_engine(args, ctx, T, R, refit_group, data_gloo):
    roles = _pd_roles(args, T, R)
    if roles is not None and ctx.rank in roles[0]:
        return run_prefill(args, ctx, T, R, refit_group, data_gloo, *roles)
    model = build_model(args, ctx)
    engine = build_engine(args, model, ctx, _overrides(args, ctx, T, R))
    tok = load_tokenizer(args)
    client = LocalEngineClient(engine, tok)
    ds_cls = load_function(args.data_source_path)
    # sample-producing ranks: every engine rank but the prefill ones
    producers = [r for r in range(T, T + R) if roles is None or r not in roles[0]]
    if roles is not None and ctx.rank in roles[1]:  # its paired prefill rank computes the prompts
        from miles_b200.rollout.pd import RemotePrefill

        pre, dec = roles
        client.remote_prefill = RemotePrefill(pre[dec.index(ctx.rank)], ctx.device)
    manager = RolloutManager(args, ds_cls(args, tok), client, tok, producers.index(ctx.rank),
                             len(producers))
    refit = make_refit(model, refit_group, src=0, bucket_bytes=args.update_weight_buffer_size,
                       mode="fp8" if args.update_weight_quant == "fp8" else "bf16",
                       transport=args.update_weight_transport)
    refit.sync()
    start, N = 0, args.num_rollout
    worker = None
    if args.fully_async:
        from miles_b200.rollout.fully_async import FullyAsyncRollout

        la = manager._local_args()
        manager.state.args = la
        worker = FullyAsyncRollout(la, manager.data_source, manager.state,
                                   lambda: model.weight_version)
    for r in range(start, N):
        if r >= start + 2 and _refit_due(r - 2, args, N, start):
            if worker is not None:
                worker.pause()
            refit.sync()
            if args.check_weight_update_equal:
                from miles_b200.parallel.refit import verify_weights_equal

                verify_weights_equal(model, refit_group, 0, args.update_weight_quant != "fp8")
            if worker is not None:
                worker.resume()
        if worker is None:
            data = manager.generate(r)
            if client.remote_prefill is not None:
                client.remote_prefill.end_step()
        else:
            groups = worker.get_batch(manager._local_args().rollout_batch_size)
            data = manager.convert_samples_to_train_data(groups)
            data["metrics"] = manager.rollout_metrics([s for g in groups for s in g], 0.0)
            data["metrics"].update(worker.metrics())
        dist.gather_object(data, None, dst=0, group=data_gloo)
    if worker is not None:
        worker.shutdown()
    return []


def train(args):
    args.fully_async = getattr(args, "fully_async", False)
    ctx, T, R, train_group, train_gloo, refit_group, data_gloo = _init(args)
    if ctx.rank < T:
        return run_trainer(args, ctx, T, train_gloo, refit_group, data_gloo)
    return run_engine(args, ctx, T, R, refit_group, data_gloo)


if __name__ == "__main__":
    hist = train(parse_args())
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
