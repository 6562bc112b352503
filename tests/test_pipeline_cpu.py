"""CPU end-to-end: tiny Qwen3-style model, rollout engine, GRPO step (plumbing config)."""
import numpy as np
import torch

from miles_b200.engine.engine import GenRequest, RolloutEngine
from miles_b200.models.config import preset
from miles_b200.models.transformer import Transformer
from miles_b200.ops.attention import VarlenMeta
from miles_b200.ops.logprob import lm_head_logprob
from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem
from miles_b200.trainer.grpo import ColocatedRL, RLConfig


def _model(name="tiny"):
    torch.manual_seed(0)
    cfg = preset(name)
    return Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)


def test_engine_greedy_matches_forward():
    m = _model()
    eng = RolloutEngine(m, max_batch=4, num_pages=64, use_cuda_graph=False)
    prompts = [[1, 2, 3, 4, 5], list(range(10, 80))]
    outs = eng.generate([GenRequest(p, 6, temperature=0.0, rid=i) for i, p in enumerate(prompts)])
    for p, o in zip(prompts, outs):
        seq = p + o.tokens
        meta = VarlenMeta([0, len(seq)], "cpu")
        with torch.no_grad():
            h = m.forward_train(torch.tensor(seq), meta)
            logits = h @ m.lm_head_weight().t()
        greedy = logits[len(p) - 1:-1].argmax(-1).tolist()
        assert greedy == o.tokens
        with torch.no_grad():
            lp, _ = lm_head_logprob(h[len(p) - 1:-1], m.lm_head_weight(), torch.tensor(o.tokens))
        assert np.allclose(lp.numpy(), o.logprobs, atol=1e-4)


def test_grpo_step_cpu():
    m = _model()
    eng = RolloutEngine(m, max_batch=32, num_pages=256, use_cuda_graph=False)
    actor = Actor(m, ActorConfig(lr=1e-3, max_tokens_per_gpu=512, grad_dtype=torch.float32))
    rl = ColocatedRL(eng, actor, RLConfig(n_samples_per_prompt=4, max_new_tokens=16))
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 4096, 64).tolist() for _ in range(8)]
    before = m.flat.clone()
    met = rl.step(prompts, rewards=rng.integers(0, 2, 32).astype(float).tolist())
    met = rl.step(prompts, rewards=rng.integers(0, 2, 32).astype(float).tolist())
    assert met["train/train_rollout_logprob_abs_diff"] < 1e-4
    assert np.isfinite(met["grad_norm"])
    assert not torch.equal(before, m.flat)
    assert m.weight_version == 2


def test_moe_engine_and_replay_cpu():
    m = _model("tiny-moe")
    eng = RolloutEngine(m, max_batch=8, num_pages=64, use_cuda_graph=False)
    out = eng.generate([GenRequest([5, 6, 7, 8], 5, temperature=1.0, seed=3,
                                   return_routed_experts=True, rid=0)])[0]
    assert out.routed_experts.shape == (4 + 5 - 1, 2, 2)
    actor = Actor(m, ActorConfig(use_routing_replay=True, grad_dtype=torch.float32))
    it = TrainItem(tokens=[5, 6, 7, 8] + out.tokens, prompt_len=4, rollout_logp=out.logprobs,
                   routed_experts=out.routed_experts)
    lp = actor.compute_logprobs([it])[0]
    assert np.allclose(lp, out.logprobs, atol=1e-4)


def test_partial_rollout_over_sampling_cpu():
    """Partial rollout: each step trains the first `groups_per_step` complete groups; the rest
    keep their partial responses and continue next step. With lr 0 the continued samples equal
    one uninterrupted generation (the sampler is a function of seed and position)."""
    m = _model("tiny-moe")
    eng = RolloutEngine(m, max_batch=16, num_pages=256, use_cuda_graph=False, steps_per_sync=2)
    actor = Actor(m, ActorConfig(lr=0.0, max_tokens_per_gpu=512, grad_dtype=torch.float32,
                                 use_routing_replay=True))
    cfg = RLConfig(n_samples_per_prompt=2, partial_rollout=True, groups_per_step=2,
                   over_sampling=2, routing_replay=True)
    rl = ColocatedRL(eng, actor, cfg)
    rng = np.random.default_rng(0)
    seen = {}
    for step in range(4):
        k = rl.prompts_needed()
        assert k == (4 if step == 0 else 2)
        prompts = [rng.integers(0, 4096, 8).tolist() for _ in range(k)]
        lens = rng.integers(2, 30, 2 * k).tolist()
        met = rl.step(prompts, lens, rng.integers(0, 2, 2 * k).astype(float).tolist())
        assert met["rollout/buffered_groups"] == 2
        for g in rl.last_groups:
            for s in g:
                assert s.response_length == s.metadata["max_new"]
                assert len(s.rollout_log_probs) == s.response_length == len(s.loss_mask)
                assert s.rollout_routed_experts.shape[0] == len(s.tokens) - 1
                seen[s.index] = s
    assert any(s.metadata.get("resumed") for s in seen.values())  # some crossed a step boundary
    # lr 0: every trained sample equals one uninterrupted generation of the same request
    for s in list(seen.values())[:6]:
        plen = s.metadata["prompt_len"]
        ref = eng.generate([GenRequest(s.tokens[:plen], s.response_length, seed=s.metadata["seed"],
                                       rid=0)])[0]
        assert ref.tokens == s.tokens[plen:]
        assert np.allclose(ref.logprobs, s.rollout_log_probs, atol=1e-5)


def test_engine_client_joins_running_batch_cpu():
    """Requests that arrive while a generate() call runs join its batch (engine.submit) instead
    of waiting for the whole wave; results equal standalone generation (same seeds)."""
    import asyncio

    from miles_b200.rollout.engine_client import LocalEngineClient

    m = _model()
    eng = RolloutEngine(m, max_batch=8, num_pages=128, use_cuda_graph=False, steps_per_sync=2)
    client = LocalEngineClient(eng)
    p1, p2 = list(range(5, 25)), list(range(40, 52))

    async def run():
        t1 = asyncio.ensure_future(client.generate(p1, {"max_new_tokens": 40, "sampling_seed": 1}))
        await asyncio.sleep(0.3)  # the first call is decoding by now
        t2 = asyncio.ensure_future(client.generate(p2, {"max_new_tokens": 6, "sampling_seed": 2}))
        return await t1, await t2

    r1, r2 = asyncio.run(run())
    assert eng.stats["prefills"] >= 1
    ref = eng.generate([GenRequest(p1, 40, seed=1, rid=0), GenRequest(p2, 6, seed=2, rid=1)])
    assert r1["output_ids"] == ref[0].tokens and r2["output_ids"] == ref[1].tokens


def test_old_logprobs_from_training_forward_cpu():
    """With one optimizer step per rollout, old log-probs taken from the training forward give
    the same update as a separate no-grad pass (same weights, same kernels)."""
    results = []
    for from_fwd in (False, True):
        m = _model()
        eng = RolloutEngine(m, max_batch=16, num_pages=256, use_cuda_graph=False)
        actor = Actor(m, ActorConfig(lr=1e-3, max_tokens_per_gpu=512, grad_dtype=torch.float32,
                                     old_logp_from_forward=from_fwd))
        rl = ColocatedRL(eng, actor, RLConfig(n_samples_per_prompt=4, max_new_tokens=8))
        rng = np.random.default_rng(1)
        prompts = [rng.integers(0, 4096, 16).tolist() for _ in range(2)]
        met = rl.step(prompts, rewards=[1.0, 0.0, 1.0, 0.0, 0.0, 1.0, 1.0, 0.0])
        results.append((m.flat.clone(), met))
    assert torch.allclose(results[0][0], results[1][0], atol=1e-6)
    assert results[1][1]["train/train_rollout_logprob_abs_diff"] < 1e-4
