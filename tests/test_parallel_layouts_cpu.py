"""Model-parallel layouts on CPU (gloo): EP alone, TP x EP with TP-split experts, TP x EP and TP
alone with whole experts (expert-tensor-parallel size 1), TP x CP (also for MLA / DSA and the
Gated DeltaNet hybrid). Each layout's groups come from
`init_distributed`; one actor step over data-parallel shards of a batch, then `save_hf`, gives
the same HF tensors as one process stepping on the whole batch; the gradient norm is the
global one on every rank."""
import argparse
import dataclasses
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import free_port

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def _cfg(variant="moe"):
    from miles_b200.models.config import preset

    # 4 KV heads: 2 per TP rank, split again over 2 CP ranks
    base = dataclasses.replace(preset("tiny-moe"), num_experts=8, num_heads=8, num_kv_heads=4)
    if variant == "biased":  # separate q / k / v with biases, half-width rotary (GLM-4.5-like)
        return dataclasses.replace(base, attention_bias=True, partial_rotary_factor=0.5)
    if variant == "mla":
        return preset("tiny-dsa")
    if variant == "gdn":  # Gated DeltaNet hybrid: states handed over along each TP rank's CP group
        return dataclasses.replace(preset("tiny-gdn"), num_heads=8, num_kv_heads=4)
    return base


def _items(cfg, n=8):
    from miles_b200.trainer.actor import TrainItem

    rng = np.random.default_rng(3)
    out = []
    for _ in range(n):
        P, R = int(rng.integers(5, 14)), int(rng.integers(3, 9))
        toks = rng.integers(0, cfg.vocab_size, P + R).tolist()
        out.append(TrainItem(toks, P, advantage=float(rng.normal()),
                             rollout_logp=(-rng.random(R)).tolist()))
    return out


def _actor_cfg():
    from miles_b200.trainer.actor import ActorConfig

    return ActorConfig(lr=1e-3, max_tokens_per_gpu=48, grad_dtype=torch.float32,
                       optimizer_placement="device")


def _run(rank, world, port, layout, ckpt, out, variant):
    os.environ.update(MILES_B200_FORCE_CPU="1", RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.transformer import Transformer
    from miles_b200.orchestration.setup import init_distributed
    from miles_b200.trainer.actor import Actor

    tp, ep, etp, cp = layout
    args = argparse.Namespace(distributed_timeout_minutes=5, tensor_model_parallel_size=tp,
                              expert_model_parallel_size=ep, context_parallel_size=cp,
                              pipeline_model_parallel_size=1, expert_tensor_parallel_size=etp)
    ctx = init_distributed(args)
    cfg = _cfg(variant)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7, tp_group=ctx.tp_group,
                    ep_group=ctx.ep_group, cp_group=ctx.cp_group, etp=etp)
    load_hf(m, ckpt)
    a = Actor(m, _actor_cfg(), dp_group=ctx.dp_group)  # as build_actor: gradients over DP x CP
    a.expert_dp_group = ctx.expert_dp_group
    items = _items(cfg)
    n_tok = sum(it.resp_len for it in items)
    mine = items[ctx.dp_rank::ctx.dp_size]
    met = a.train_step(mine, global_num_samples=len(items), global_num_tokens=n_tok)
    if ctx.cp_group is not None:
        saver = ctx.dp_rank == 0 and dist.get_rank(ctx.cp_group) == 0
    else:
        saver = rank < (tp * ep if (etp or tp) > 1 else max(tp, ep))
    if saver:
        save_hf(m, out)
    torch.save(met["grad_norm"], f"{out}.gn{rank}")
    dist.destroy_process_group()


@pytest.mark.parametrize("layout,world,port", [
    ((1, 2, None, 1), 2, 29691),     # EP2
    ((2, 2, None, 1), 4, 29692),     # TP2 x EP2, experts split over TP
    ((2, 2, 1, 1), 4, 29693),        # TP2 x EP2, whole experts (EP group = TP group)
    ((2, 1, 1, 1), 2, 29694),        # TP2, whole experts on both ranks
    ((2, 1, None, 2), 4, 29695),     # TP2 x CP2
    ((2, 1, None, 2, "biased"), 4, 29696),   # TP2 x CP2, separate biased q / k / v
    ((2, 1, None, 2, "mla"), 4, 29698),      # TP2 x CP2, MLA + DSA
    ((2, 1, None, 2, "gdn"), 4, 29699),      # TP2 x CP2, Gated DeltaNet hybrid
])
def test_layouts_match_single(tmp_path, layout, world, port):
    from safetensors import safe_open

    from miles_b200.checkpoint.hf import save_hf, to_hf_tensors
    from miles_b200.models.transformer import Transformer
    from miles_b200.trainer.actor import Actor

    variant = layout[4] if len(layout) > 4 else "moe"
    layout = layout[:4]
    cfg = _cfg(variant)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7)
    ckpt = str(tmp_path / "hf")
    save_hf(m, ckpt)
    a = Actor(m, _actor_cfg())
    met = a.train_step(_items(cfg))
    from miles_b200.checkpoint.hf import to_hf_layout

    # compared in the saved (HF) layout: zero-centred norms and the conv weight differ from ours
    ref = {k: to_hf_layout(cfg, k, v.detach()).clone() for k, v in to_hf_tensors(m)}
    out = str(tmp_path / "out")
    mp.spawn(_run, args=(world, free_port(), layout, ckpt, out, variant), nprocs=world, join=True)
    import json

    wm = json.load(open(os.path.join(out, "model.safetensors.index.json")))["weight_map"]
    assert set(wm) == set(ref), set(ref) ^ set(wm)
    bad = []
    for name, fn in wm.items():
        with safe_open(os.path.join(out, fn), "pt") as f:
            got = f.get_tensor(name)
        if not torch.allclose(got, ref[name], atol=2e-5):
            bad.append((name, float((got - ref[name]).abs().max())))
    assert not bad, bad
    for r in range(world):
        gn = torch.load(f"{out}.gn{r}")
        assert abs(gn - met["grad_norm"]) < 1e-4 * max(1.0, met["grad_norm"]), (r, gn, met["grad_norm"])
