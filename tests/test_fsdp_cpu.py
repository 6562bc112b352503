"""FSDP2 training backend on CPU (gloo): a 2-rank fully sharded step over half the samples per
rank gives the parameters of a one-process step over all samples; the gathered HF state loads
into this framework's Transformer (the rollout engine's model) with equal logits."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")
pytest.importorskip("transformers")


def _items():
    from miles_b200.trainer.actor import TrainItem

    rng = np.random.default_rng(0)
    out = []
    for i in range(4):
        P, R = int(rng.integers(4, 12)), int(rng.integers(3, 9))
        out.append(TrainItem(rng.integers(0, 256, P + R).tolist(), P, advantage=float(rng.normal()),
                             rollout_logp=(-rng.random(R)).tolist()))
    return out


def _cfg():
    from miles_b200.ops.rl import PolicyLossCfg
    from miles_b200.trainer.actor import ActorConfig

    return ActorConfig(lr=1e-3, loss=PolicyLossCfg(eps_clip=0.2, eps_clip_high=0.2), max_tokens_per_gpu=64)


def _step(actor, items, n_global):
    old = actor.compute_logprobs(items)
    for it, o in zip(items, old):
        it.old_logp = o
    return actor.train_step(items, global_num_samples=n_global)


def _rank(rank, port, ckpt, out):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    from miles_b200.trainer.fsdp_actor import FSDPActor

    actor = FSDPActor(ckpt, _cfg())
    items = _items()[rank::2]
    m = _step(actor, items, 4)
    state = actor.export_hf_state()
    if rank == 0:
        torch.save({"state": state, "metrics": m}, out)
    dist.barrier()
    dist.destroy_process_group()


def test_fsdp2_step_matches_single_process(tmp_path):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from miles_b200.checkpoint.hf import load_hf_tensors
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.trainer.fsdp_actor import FSDPActor

    torch.manual_seed(0)
    hf = Qwen3ForCausalLM(Qwen3Config(vocab_size=256, hidden_size=128, intermediate_size=256,
                                      num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                                      head_dim=32, tie_word_embeddings=False))
    ckpt = str(tmp_path / "hf")
    hf.save_pretrained(ckpt)
    single = FSDPActor(ckpt, _cfg())
    m1 = _step(single, _items(), 4)
    ref = single.export_hf_state()
    out = str(tmp_path / "r.pt")
    mp.spawn(_rank, args=(free_port(), ckpt, out), nprocs=2, join=True)
    r = torch.load(out)
    assert abs(r["metrics"]["grad_norm"] - m1["grad_norm"]) < 1e-4 * max(1.0, m1["grad_norm"])
    for k, v in ref.items():
        assert torch.allclose(r["state"][k], v, atol=1e-5, rtol=1e-4), k
    # the trained HF state feeds this framework's model (the engine side of a refit)
    cfg = ModelConfig.from_hf(ckpt)
    mine = Transformer(cfg, device="cpu", dtype=torch.float32, materialize=False)
    load_hf_tensors(mine, r["state"])
    toks = torch.randint(0, 256, (1, 21))
    with torch.no_grad():
        want = single.hf(toks).logits[0].float()
        got = mine.forward_train(toks[0].int(), VarlenMeta([0, 21], "cpu")).float() @ mine.lm_head_weight().float().t()
    assert (want - got).abs().max() < 1e-4 * max(1.0, want.abs().max().item())


@pytest.mark.timeout(600)
def test_train_fsdp_backend(tmp_path):
    """train.py --train-backend fsdp on 2 gloo ranks: rollout by this framework's engine,
    training of the HF policy under FSDP2, engine weights refreshed after each step."""
    import json
    import subprocess
    import sys

    from transformers import Qwen3Config, Qwen3ForCausalLM

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    torch.manual_seed(0)
    Qwen3ForCausalLM(Qwen3Config(vocab_size=256, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                                 num_attention_heads=4, num_key_value_heads=2, head_dim=32,
                                 tie_word_embeddings=False)).save_pretrained(str(tmp_path / "hf"))
    rng = np.random.default_rng(0)
    with open(tmp_path / "d.jsonl", "w") as f:
        for _ in range(4):
            f.write(json.dumps({"input": rng.integers(0, 256, 12).tolist(), "label": "1"}) + "\n")
    env = dict(os.environ, MILES_B200_FORCE_CPU="1", PYTHONPATH=root, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), os.path.join(root, "train.py"),
           "--hf-checkpoint", str(tmp_path / "hf"), "--train-backend", "fsdp",
           "--prompt-data", str(tmp_path / "d.jsonl"), "--label-key", "label",
           "--rollout-batch-size", "2", "--n-samples-per-prompt", "2", "--rollout-max-response-len", "8",
           "--rm-type", "random", "--num-rollout", "2", "--lr", "1e-3", "--max-tokens-per-gpu", "256",
           "--actor-num-gpus-per-node", "2", "--ci-test"]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=580)
    assert r.returncode == 0, r.stderr[-3000:]
