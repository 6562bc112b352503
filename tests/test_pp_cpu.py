"""Pipeline parallelism on CPU (gloo): a PP2 / PP3 actor step over several micro-batches (1F1B)
gives the same old log-probs, metrics and updated parameters as one rank, tied embeddings
included; train.py runs with --pipeline-model-parallel-size 2."""
import dataclasses
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _items(cfg, n=5):
    from miles_b200.trainer.actor import TrainItem

    rng = np.random.default_rng(1)
    out = []
    for i in range(n):
        P, R = int(rng.integers(5, 20)), int(rng.integers(3, 12))
        toks = rng.integers(0, cfg.vocab_size, P + R).tolist()
        out.append(TrainItem(toks, P, advantage=float(rng.normal()),
                             rollout_logp=(-rng.random(R)).tolist()))
    return out


def _actor(model):
    from miles_b200.trainer.actor import Actor, ActorConfig

    # small token budget: several micro-batches go through the pipeline
    return Actor(model, ActorConfig(lr=1e-3, max_tokens_per_gpu=40, grad_dtype=torch.float32,
                                    optimizer_placement="device"))


def _step(model, cfg):
    a = _actor(model)
    items = _items(cfg)
    old = a.compute_logprobs(items)
    for it, o in zip(items, old):
        it.old_logp = o
    m = a.train_step(items)
    return old, m


def _run(rank, world, port, name, ckpt, out):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from miles_b200.checkpoint.hf import load_hf
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = preset(name)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7, pp_group=dist.group.WORLD)
    load_hf(m, ckpt)
    old, met = _step(m, cfg)
    torch.save({"old": old, "metrics": met, "params": {k: v.detach().clone() for k, v in m.params.items()}},
               f"{out}.{rank}")
    dist.destroy_process_group()


@pytest.mark.parametrize("name,world,port", [("tiny", 2, 29661), ("tiny-moe", 2, 29662)])
def test_pp_matches_single(tmp_path, name, world, port):
    from miles_b200.checkpoint.hf import save_hf
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = preset(name)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7)
    ckpt = str(tmp_path / "hf")
    save_hf(m, ckpt)
    old1, met1 = _step(m, cfg)
    out = str(tmp_path / "pp")
    mp.spawn(_run, args=(world, free_port(), name, ckpt, out), nprocs=world, join=True)
    seen = set()
    for r in range(world):
        res = torch.load(f"{out}.{r}", weights_only=False)
        for a, b in zip(res["old"], old1):
            assert np.abs(a - b).max() < 1e-5
        for k in ("pg_loss", "grad_norm"):
            if k in met1:
                assert abs(res["metrics"][k] - met1[k]) < 1e-4 * max(1.0, abs(met1[k])), (k, res["metrics"][k], met1[k])
        for k, v in res["params"].items():
            assert torch.allclose(v, m.params[k].detach(), atol=1e-5), (r, k, (v - m.params[k]).abs().max())
            seen.add(k)
    assert seen == set(m.params)


@pytest.mark.timeout(600)
def test_train_pp2(tmp_path):
    rng = np.random.default_rng(0)
    with open(tmp_path / "d.jsonl", "w") as f:
        for _ in range(8):
            f.write(json.dumps({"input": rng.integers(0, 4096, 64).tolist(), "label": "1"}) + "\n")
    env = dict(os.environ, MILES_B200_FORCE_CPU="1", PYTHONPATH=ROOT, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), os.path.join(ROOT, "train.py"),
           "--model-name", "tiny", "--prompt-data", str(tmp_path / "d.jsonl"), "--label-key", "label",
           "--rollout-batch-size", "4", "--n-samples-per-prompt", "4", "--rollout-max-response-len", "16",
           "--rm-type", "random", "--num-rollout", "2", "--lr", "1e-3", "--max-tokens-per-gpu", "128",
           "--actor-num-gpus-per-node", "2", "--pipeline-model-parallel-size", "2", "--ci-test",
           "--save", str(tmp_path / "ckpt"), "--save-interval", "1",
           "--save-hf", str(tmp_path / "hf_{rollout_id}")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=580)
    assert r.returncode == 0, r.stderr[-3000:]
    idx = json.load(open(tmp_path / "hf_1" / "model.safetensors.index.json"))["weight_map"]
    assert "model.layers.0.mlp.down_proj.weight" in idx and "model.layers.1.mlp.down_proj.weight" in idx


def test_interleaved_schedule_plan():
    """Every op of every rank runs exactly once, after its inputs, and interleaving shrinks the
    pipeline bubble ((P - 1) / V stage-times instead of P - 1)."""
    from miles_b200.parallel.pp import interleaved_schedule

    for P, V, n in [(2, 2, 4), (4, 2, 8), (4, 4, 8), (3, 2, 5), (2, 3, 7), (2, 2, 1)]:
        plan = interleaved_schedule(P, V, n)
        when = {}
        for t, (ops, msgs) in enumerate(plan):
            for s, (kind, j, c) in ops.items():
                key = (kind, j, c * P + s)
                assert key not in when
                when[key] = t
            for src, dst, kind, j, vd in msgs:
                assert vd % P == dst and (vd + (1 if kind == "B" else -1)) % P == src
        NV = P * V
        assert len(when) == 2 * n * NV
        for (kind, j, v), t in when.items():
            if kind == "F" and v > 0:
                assert when[("F", j, v - 1)] < t
            if kind == "B":
                assert when[("F", j, v)] < t
                if v < NV - 1:
                    assert when[("B", j, v + 1)] < t
    # bubble: P=4, 8 micro-batches; ticks are chunk-times (1/V of a stage-time)
    t1 = len(interleaved_schedule(4, 1, 8))
    t2 = len(interleaved_schedule(4, 2, 8)) / 2
    assert t2 < t1
    fo = interleaved_schedule(2, 2, 3, train=False)
    assert all(op[0] == "F" for ops, _ in fo for op in ops.values())


def _run_vpp(rank, world, port, name, ckpt, out, vpp, first=None, last=None):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from miles_b200.checkpoint.hf import load_hf
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = dataclasses.replace(preset(name), num_layers=4)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7, pp_group=dist.group.WORLD, vpp=vpp,
                    pp_first_layers=first, pp_last_layers=last)
    assert len(m.pp.chunks) == vpp
    load_hf(m, ckpt)
    old, met = _step(m, cfg)
    torch.save({"old": old, "metrics": met, "params": {k: v.detach().clone() for k, v in m.params.items()}},
               f"{out}.{rank}")
    dist.destroy_process_group()


@pytest.mark.parametrize("name,world,vpp,port,first,last", [
    ("tiny", 2, 2, 29663, None, None), ("tiny-moe", 2, 2, 29664, None, None),
    ("tiny", 2, 1, 29665, 1, 3)])
def test_interleaved_pp_matches_single(tmp_path, name, world, vpp, port, first, last):
    """Interleaved (virtual) pipeline: each of 2 ranks holds 2 model chunks (4 layers -> virtual
    stages of one layer, rank 0 layers {0, 2}, rank 1 layers {1, 3}); the step equals one rank's."""
    from miles_b200.checkpoint.hf import save_hf
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = dataclasses.replace(preset(name), num_layers=4)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=7)
    ckpt = str(tmp_path / "hf")
    save_hf(m, ckpt)
    old1, met1 = _step(m, cfg)
    out = str(tmp_path / "vpp")
    mp.spawn(_run_vpp, args=(world, free_port(), name, ckpt, out, vpp, first, last), nprocs=world, join=True)
    seen = set()
    for r in range(world):
        res = torch.load(f"{out}.{r}", weights_only=False)
        for a, b in zip(res["old"], old1):
            assert np.abs(a - b).max() < 1e-5
        for k in ("pg_loss", "grad_norm"):
            if k in met1:
                assert abs(res["metrics"][k] - met1[k]) < 1e-4 * max(1.0, abs(met1[k])), (k, res["metrics"][k], met1[k])
        for k, v in res["params"].items():
            assert torch.allclose(v, m.params[k].detach(), atol=1e-5), (r, k, (v - m.params[k]).abs().max())
            seen.add(k)
    assert seen == set(m.params)


def test_stage_layer_counts():
    from miles_b200.parallel.pp import stage_layer_counts

    assert stage_layer_counts(10, 4) == [3, 3, 2, 2]
    assert stage_layer_counts(10, 4, first=1) == [1, 3, 3, 3]
    assert stage_layer_counts(10, 4, first=1, last=2) == [1, 4, 3, 2]
    assert stage_layer_counts(4, 2, first=1, last=3) == [1, 3]
    with pytest.raises(ValueError):
        stage_layer_counts(4, 2, first=1, last=1)
