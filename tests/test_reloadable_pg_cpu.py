"""Reloadable process groups on CPU (gloo, 4 ranks, TP2 x DP2): destroying the training-only
groups between steps and rebuilding them rebinds every holder (context, model, actor) to the
new groups, keeps the TP groups, and the next step gives the same parameters as a run that
kept its groups."""
import argparse
import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def _run(rank, world, port, reload, out):
    os.environ.update(MILES_B200_FORCE_CPU="1", RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.orchestration.setup import init_distributed
    from miles_b200.parallel.reloadable import REGISTRY
    from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem

    args = argparse.Namespace(distributed_timeout_minutes=5, tensor_model_parallel_size=2,
                              expert_model_parallel_size=1, context_parallel_size=1,
                              pipeline_model_parallel_size=1, expert_tensor_parallel_size=None)
    ctx = init_distributed(args)
    cfg = preset("tiny")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7, tp_group=ctx.tp_group)
    a = Actor(m, ActorConfig(lr=1e-3, grad_dtype=torch.float32, optimizer_placement="device"),
              dp_group=ctx.dp_group)
    rng = np.random.default_rng(ctx.dp_rank)
    items = [TrainItem(rng.integers(0, cfg.vocab_size, 14).tolist(), 6, advantage=float(rng.normal()),
                       rollout_logp=(-rng.random(8)).tolist()) for _ in range(3)]
    a.train_step(items, global_num_samples=6, global_num_tokens=48)
    if reload:
        old_dp, old_tp = ctx.dp_group, ctx.tp_group
        assert REGISTRY.destroy() == 1  # this rank's DP group; the TP group is kept
        REGISTRY.reload([ctx, m, a])
        assert ctx.dp_group is not old_dp and a.dp_group is ctx.dp_group
        assert ctx.tp_group is old_tp and m.tp.group is old_tp
        assert a.opt.group is ctx.dp_group  # the sharded optimizer rebound too
        dist.barrier(group=ctx.dp_group)  # the new group works
    a.train_step(items, global_num_samples=6, global_num_tokens=48)
    torch.save({k: v.detach().clone() for k, v in m.params.items()}, f"{out}.{rank}")
    dist.destroy_process_group()


def test_reload_groups_between_steps(tmp_path):
    a, b = str(tmp_path / "keep"), str(tmp_path / "reload")
    mp.spawn(_run, args=(4, free_port(), False, a), nprocs=4, join=True)
    mp.spawn(_run, args=(4, free_port(), True, b), nprocs=4, join=True)
    for r in range(4):
        pa, pb = torch.load(f"{a}.{r}"), torch.load(f"{b}.{r}")
        for k in pa:
            assert torch.equal(pa[k], pb[k]), (r, k)
