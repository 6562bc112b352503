"""Multi-token prediction training on CPU: the MTP loss of packed sequences equals the sum over
the sequences run alone (nothing leaks across sequence boundaries), training steps lower it
and update the MTP layers, and HF / torch_dist checkpoints carry the MTP parameters under the
DeepSeek-V3 / Megatron names."""
import dataclasses
import os

import numpy as np
import pytest
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def _model(name, mtp, seed=5):
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = dataclasses.replace(preset(name), mtp_num_layers=mtp)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=seed)
    m.mtp_train = True
    return m


def _items(cfg, n=4, seed=0):
    from miles_b200.trainer.actor import TrainItem

    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        P, R = int(rng.integers(4, 9)), int(rng.integers(6, 12))
        out.append(TrainItem(rng.integers(0, cfg.vocab_size, P + R).tolist(), P, advantage=0.0,
                             rollout_logp=(-rng.random(R)).tolist()))
    return out


def _mtp_of(m, items):
    from miles_b200.trainer.actor import Actor, ActorConfig

    a = Actor(m, ActorConfig(mtp_loss_scale=1.0, grad_dtype=torch.float32, optimizer_placement="device"))
    prep = a._mb_prepare(items, len(items), sum(it.resp_len for it in items))
    m.selected_logprob(prep["tok"], prep["meta"], prep["sel"], prep["tgt"], 1.0, 4096)
    return float(m.mtp_loss(prep["tok"], prep["meta"], prep["sel"], prep["tgt"], prep["wgt"]))


@pytest.mark.parametrize("name,mtp", [("tiny", 2), ("tiny-mla", 1)])
def test_mtp_packing_isolated(name, mtp):
    m = _model(name, mtp)
    items = _items(m.cfg)
    n = len(items)
    packed = _mtp_of(m, items)
    # alone: the weights are normalised per sample over the batch, so rescale by 1 / n
    alone = sum(_mtp_of(m, [it]) for it in items) / n
    assert abs(packed - alone) < 1e-5 * max(1.0, abs(packed)), (packed, alone)


def test_mtp_training_lowers_loss():
    from miles_b200.trainer.actor import Actor, ActorConfig

    m = _model("tiny", 1)
    before = {k: v.detach().clone() for k, v in m.params.items() if ".2." in k}  # the MTP layer
    a = Actor(m, ActorConfig(lr=3e-3, mtp_loss_scale=1.0, grad_dtype=torch.float32,
                             optimizer_placement="device"))
    items = _items(m.cfg)
    losses = [a.train_step(items)["mtp_loss"] for _ in range(6)]
    assert all(np.isfinite(losses)) and losses[-1] < losses[0], losses
    assert all(not torch.equal(before[k], m.params[k]) for k in before if k.endswith(("eh_proj.weight",
                                                                                       "o_proj.weight")))


def test_mtp_checkpoints(tmp_path):
    import json

    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.checkpoint.torch_dist import model_state_dict

    m = _model("tiny-mla", 1)
    L = m.cfg.num_layers
    save_hf(m, str(tmp_path))
    idx = json.load(open(tmp_path / "model.safetensors.index.json"))["weight_map"]
    assert f"model.layers.{L}.eh_proj.weight" in idx and f"model.layers.{L}.shared_head.norm.weight" in idx
    assert json.load(open(tmp_path / "config.json"))["num_nextn_predict_layers"] == 1
    m2 = _model("tiny-mla", 1, seed=9)
    load_hf(m2, str(tmp_path))
    for k, v in m.params.items():
        assert torch.equal(v, m2.params[k]), k
    keys = set(model_state_dict(m))
    assert "mtp.layers.0.eh_proj.weight" in keys and "mtp.layers.0.final_layernorm.weight" in keys
    assert any(k.startswith("mtp.layers.0.transformer_layer.") for k in keys)


def test_mtp_rejected_on_gated_deltanet_hybrid():
    from miles_b200.models.config import preset

    cfg = dataclasses.replace(preset("tiny-gdn"), mtp_num_layers=1)
    # MTP depths numbered past the main stack are never linear-attention layers
    assert not cfg.layer_is_linear(cfg.num_layers)
    with pytest.raises(ValueError, match="Gated DeltaNet"):
        _model("tiny-gdn", 1)


def test_mtp_kept_when_base_checkpoint_has_none(tmp_path):
    from miles_b200.checkpoint.hf import load_hf, save_hf

    base = _model("tiny", 0, seed=3)
    save_hf(base, str(tmp_path))
    m = _model("tiny", 1, seed=9)
    before = m.p("layers.%d.eh_proj.weight" % m.cfg.num_layers).clone()
    with pytest.warns(UserWarning, match="multi-token prediction"):
        load_hf(m, str(tmp_path))
    assert torch.equal(m.p("layers.0.mlp.down_proj.weight"), base.p("layers.0.mlp.down_proj.weight"))
    assert torch.equal(m.p("layers.%d.eh_proj.weight" % m.cfg.num_layers), before)


def test_mtp_depth_from_hf_config():
    from miles_b200.models.config import ModelConfig

    c = ModelConfig.from_hf({"model_type": "qwen3", "vocab_size": 64, "hidden_size": 32,
                             "num_hidden_layers": 2, "num_attention_heads": 2,
                             "num_nextn_predict_layers": 2})
    assert c.extra["num_nextn_predict_layers"] == 2
