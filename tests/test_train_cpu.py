"""CPU end-to-end of train.py (the plumbing configuration): tiny Qwen3-style model, GRPO,
single process and a 2-rank gloo world; checkpoint save/resume round trip."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
from tests.conftest import free_port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _dataset(path, n=8, L=64, vocab=4096, seed=0):
    rng = np.random.default_rng(seed)
    with open(path, "w") as f:
        for i in range(n):
            f.write(json.dumps({"input": rng.integers(0, vocab, L).tolist(), "label": "1"}) + "\n")


def _argv(tmp, extra=()):
    return ["--model-name", "tiny", "--prompt-data", str(tmp / "d.jsonl"), "--label-key", "label",
            "--rollout-batch-size", "4", "--n-samples-per-prompt", "4", "--rollout-max-response-len", "16",
            "--rm-type", "random", "--num-rollout", "2", "--lr", "1e-3", "--max-tokens-per-gpu", "1024",
            "--actor-num-gpus-per-node", "1", "--ci-test", "--save", str(tmp / "ckpt"), "--save-interval", "1",
            *extra]


def test_train_single_process(tmp_path, monkeypatch):
    monkeypatch.setenv("MILES_B200_FORCE_CPU", "1")
    _dataset(tmp_path / "d.jsonl")
    sys.path.insert(0, ROOT)
    import train as T
    from miles_b200.utils.arguments import parse_args
    from miles_b200.rollout.default import GenerateState

    GenerateState._inst = None
    hist = T.train(parse_args(_argv(tmp_path)))
    assert len(hist) == 2
    assert hist[0]["train/train_rollout_logprob_abs_diff"] < 1e-4
    assert os.path.exists(tmp_path / "ckpt" / "latest_checkpointed_iteration.txt")
    # resume from the checkpoint: starts at rollout 2 and runs one more
    GenerateState._inst = None
    hist2 = T.train(parse_args(_argv(tmp_path, ["--load", str(tmp_path / "ckpt"), "--num-rollout", "3"])))
    assert [h["step"] for h in hist2] == [2]


@pytest.mark.timeout(600)
def test_train_gloo_world2(tmp_path):
    _dataset(tmp_path / "d.jsonl")
    env = dict(os.environ, MILES_B200_FORCE_CPU="1", PYTHONPATH=ROOT, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()), os.path.join(ROOT, "train.py"),
           *_argv(tmp_path, ["--actor-num-gpus-per-node", "2", "--num-rollout", "1"])]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=580)
    assert r.returncode == 0, r.stderr[-3000:]


@pytest.mark.timeout(900)
def test_train_tp2(tmp_path):
    """Tensor parallel 2 (both ranks one TP group): two GRPO steps with torch_dist saves, then a
    resume from the TP-sharded checkpoint and an HF export gathered over the TP group."""
    _dataset(tmp_path / "d.jsonl")
    env = dict(os.environ, MILES_B200_FORCE_CPU="1", PYTHONPATH=ROOT, OMP_NUM_THREADS="2")
    base = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
            "--master-addr", "127.0.0.1", "--master-port", str(free_port()), os.path.join(ROOT, "train.py")]
    tp = ["--actor-num-gpus-per-node", "2", "--tensor-model-parallel-size", "2"]
    r = subprocess.run(base + _argv(tmp_path, tp), env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stderr[-3000:]
    r = subprocess.run(base + _argv(tmp_path, tp + ["--load", str(tmp_path / "ckpt"), "--num-rollout", "3",
                                                    "--save-hf", str(tmp_path / "hf_{rollout_id}")]),
                       env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stderr[-3000:]
    assert os.path.exists(tmp_path / "hf_2" / "model.safetensors.index.json")


def _async_run(tmp_path, extra, port, rollout_gpus: int = 1):
    _dataset(tmp_path / "d.jsonl")
    env = dict(os.environ, MILES_B200_FORCE_CPU="1", PYTHONPATH=ROOT, OMP_NUM_THREADS="2")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={1 + rollout_gpus}",
           "--master-addr", "127.0.0.1", "--master-port", str(port),
           os.path.join(ROOT, "train_async.py"),
           *_argv(tmp_path, ["--actor-num-gpus-per-node", "1", "--rollout-num-gpus", str(rollout_gpus),
                             "--num-rollout", "3", "--save-interval", "100", *extra])]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=580)
    assert r.returncode == 0, r.stderr[-3000:]
    return r


@pytest.mark.timeout(600)
def test_train_async_disaggregated(tmp_path):
    """1 trainer + 1 rollout rank: one-step-ahead pipeline with bf16 broadcast refits."""
    _async_run(tmp_path, ["--check-weight-update-equal"], free_port())


@pytest.mark.timeout(600)
def test_train_async_prefill_decode_disaggregation(tmp_path):
    """1 trainer + 1 prefill rank + 1 decode rank (--prefill-num-servers 1): the decode rank's
    requests are prefilled on its paired rank and decoded from the hand-offs; both engine ranks
    take the refits."""
    r = _async_run(tmp_path, ["--prefill-num-servers", "1", "--check-weight-update-equal"], free_port(),
                   rollout_gpus=2)
    served = [int(line.split("prefilled ")[1].split()[0]) for line in r.stdout.splitlines()
              if "prefilled" in line]
    assert len(served) == 3 and all(n > 0 for n in served), r.stdout[-2000:]


@pytest.mark.timeout(600)
def test_train_async_deployment_yaml_prefill_decode(tmp_path):
    """--sglang-config with a prefill and a decode group (and engine overrides): the same
    disaggregated loop as --prefill-num-servers, set up from the deployment file."""
    (tmp_path / "dep.yaml").write_text(
        "sglang:\n  - name: actor\n    update_weights: true\n    server_groups:\n"
        "      - {worker_type: prefill, num_gpus: 1, overrides: {max_running_requests: 16}}\n"
        "      - {worker_type: decode, num_gpus: 1}\n")
    r = _async_run(tmp_path, ["--sglang-config", str(tmp_path / "dep.yaml")], free_port(),
                   rollout_gpus=2)
    served = [int(line.split("prefilled ")[1].split()[0]) for line in r.stdout.splitlines()
              if "prefilled" in line]
    assert len(served) == 3 and all(n > 0 for n in served), r.stdout[-2000:]


def test_deployment_helpers(tmp_path):
    import types

    import pytest as _pt

    from miles_b200.rollout.sglang_config import load_deployment, overrides_for, pd_pairs

    (tmp_path / "a.yaml").write_text(
        "sglang:\n  - name: actor\n    server_groups:\n"
        "      - {worker_type: regular, num_gpus: 2, overrides: {mem_fraction_static: 0.5}}\n"
        "      - {worker_type: prefill, num_gpus: 1}\n      - {worker_type: decode, num_gpus: 1}\n")
    args = types.SimpleNamespace(sglang_config=str(tmp_path / "a.yaml"), hf_checkpoint=None,
                                 rollout_num_gpus_per_engine=1)
    engines, _ = load_deployment(args, [4, 5, 6, 7])
    assert overrides_for(engines, 5) == {"mem_fraction_static": 0.5} and overrides_for(engines, 6) == {}
    assert pd_pairs(engines) == ([6], [7])
    with _pt.raises(ValueError):
        load_deployment(args, [0, 1, 2])


@pytest.mark.timeout(600)
def test_train_async_fully_async_fp8_refit(tmp_path):
    """Continuous generation worker (partial rollout, staleness filter) and fp8 refits."""
    _async_run(tmp_path, ["--fully-async", "--partial-rollout", "--max-weight-staleness", "4",
                          "--update-weight-quant", "fp8", "--check-weight-update-equal"], free_port())


def test_train_ppo_with_critic(tmp_path, monkeypatch):
    """--advantage-estimator ppo: critic values -> GAE advantages -> value + policy updates."""
    monkeypatch.setenv("MILES_B200_FORCE_CPU", "1")
    _dataset(tmp_path / "d.jsonl")
    sys.path.insert(0, ROOT)
    import train as T
    from miles_b200.utils.arguments import parse_args
    from miles_b200.rollout.default import GenerateState

    GenerateState._inst = None
    hist = T.train(parse_args(_argv(tmp_path, ["--advantage-estimator", "ppo", "--save-interval", "100",
                                               "--ci-disable-kl-checker"])))
    assert len(hist) == 2
    assert all("critic/value_loss" in h for h in hist)
    assert np.isfinite(hist[-1]["critic/value_loss"])


def test_train_lora(tmp_path, monkeypatch):
    """--lora-rank: base weights frozen, adapters trained, rollout uses the adapters (on-policy
    log-probs stay equal), adapter checkpoint round trip."""
    monkeypatch.setenv("MILES_B200_FORCE_CPU", "1")
    _dataset(tmp_path / "d.jsonl")
    sys.path.insert(0, ROOT)
    import torch
    import train as T
    from miles_b200.utils.arguments import parse_args
    from miles_b200.rollout.default import GenerateState

    GenerateState._inst = None
    args = parse_args(_argv(tmp_path, ["--lora-rank", "4", "--lora-alpha", "8",
                                       "--target-modules", "all-linear"]))
    ctx, model, actor, engine, manager, trainer, tracker, start, ds = T.setup(args)
    base = model.flat.clone()
    data = manager.generate(0)
    m = trainer.train(0, data)
    assert torch.equal(base, model.flat)  # frozen base
    assert any(float(b.abs().sum()) > 0 for b in model.lora.B.values())
    data = manager.generate(1)  # engine now decodes with non-zero adapters
    m = trainer.train(1, data)
    assert m["train/train_rollout_logprob_abs_diff"] < 1e-4
    from miles_b200.checkpoint.torch_dist import load_checkpoint, save_checkpoint

    save_checkpoint(str(tmp_path / "ck"), 1, model, actor.opt)
    saved = {k: v.clone() for k, v in model.lora.state_dict().items()}
    for b in model.lora.B.values():
        b.data.zero_()
    load_checkpoint(str(tmp_path / "ck"), model, actor.opt)
    for k, v in model.lora.state_dict().items():
        assert torch.equal(v, saved[k])
