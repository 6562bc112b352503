"""GPU end-to-end: engine (CUDA graphs) + trainer on the sm_100a kernels, small shapes."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["small-moe", "qwen3-small"])
def test_grpo_step_bitwise_logprobs(name):
    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.models.config import ModelConfig, preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops import check_device_error
    from miles_b200.ops.rl import PolicyLossCfg
    from miles_b200.trainer.actor import Actor, ActorConfig
    from miles_b200.trainer.grpo import ColocatedRL, RLConfig

    if name == "qwen3-small":
        cfg = ModelConfig(arch="qwen3", vocab_size=8192, hidden_size=512, num_layers=2, num_heads=8,
                          num_kv_heads=2, head_dim=128, intermediate_size=1024, max_position=8192)
    else:
        cfg = preset(name)
    model = Transformer(cfg, device="cuda", seed=0)
    eng = RolloutEngine(model, max_batch=16, num_pages=256)
    actor = Actor(model, ActorConfig(lr=1e-5, max_tokens_per_gpu=1024,
                                     loss=PolicyLossCfg(use_tis=True, tis_clip=2.0),
                                     use_routing_replay=cfg.is_moe))
    rl = ColocatedRL(eng, actor, RLConfig(n_samples_per_prompt=4, routing_replay=cfg.is_moe))
    rng = np.random.default_rng(0)
    for step in range(2):
        prompts = [rng.integers(0, cfg.vocab_size, int(rng.integers(20, 150))).tolist() for _ in range(4)]
        lens = rng.integers(10, 90, 16).tolist()
        m = rl.step(prompts, lens, rewards=rng.integers(0, 2, 16).astype(float).tolist())
        # trainer log-probs equal the engine's bit for bit (CUDA-graph decode vs packed forward)
        assert m["train/train_rollout_logprob_abs_diff"] == 0.0, m
        assert np.isfinite(m["grad_norm"]) and m["grad_norm"] > 0
    torch.cuda.synchronize()
    check_device_error()
