"""CPU tests: CLI surface + validation, reward graders, data sources and filters."""
import json
import os

import pytest

from miles_b200.rollout import rm_hub
from miles_b200.rollout.data import RolloutDataSourceWithBuffer
from miles_b200.rollout.filter_hub import check_reward_nonzero_std
from miles_b200.utils.arguments import parse_args
from miles_b200.utils.types import Sample


def test_parse_defaults_and_validation():
    a = parse_args(["--rollout-batch-size", "8", "--n-samples-per-prompt", "4", "--colocate",
                    "--actor-num-gpus-per-node", "2", "--sglang-mem-fraction-static", "0.7",
                    "--use-rollout-routing-replay", "--advantage-estimator", "ppo"])
    assert a.eps_clip_high == a.eps_clip == 0.2
    assert a.over_sampling_batch_size == 8
    assert a.offload_train and a.offload_rollout and a.rollout_num_gpus == 2
    assert a.use_routing_replay and a.use_critic
    assert a.sglang_args["mem_fraction_static"] == "0.7"
    assert a.global_batch_size == 32
    assert a.tis_clip == 2.0 and a.update_weight_buffer_size == 512 * 1024 ** 2


def test_validation_errors():
    with pytest.raises(ValueError):
        parse_args(["--rollout-batch-size", "8", "--over-sampling-batch-size", "4"])
    with pytest.raises(ValueError):
        parse_args(["--colocate", "--update-weight-transfer-mode", "p2p"])
    with pytest.raises(SystemExit):
        parse_args(["--no-such-flag"])


def test_graders():
    assert rm_hub.last_boxed(r"so \boxed{\frac{1}{2}} done") == r"\frac{1}{2}"
    assert rm_hub.grade_answer(r"answer \boxed{0.5}", "1/2")
    assert rm_hub.grade_answer(r"\boxed{ 12 }", "12")
    assert not rm_hub.grade_answer(r"\boxed{13}", "12")
    assert rm_hub.deepscaler_reward(r"<think>x</think> \boxed{3}", "3") == 1
    assert rm_hub.deepscaler_reward(r"<think>x \boxed{3}", "3") == 0
    d = rm_hub.dapo_reward("work...\nAnswer: 42", "42")
    assert d["score"] == 1.0 and d["acc"]
    assert rm_hub.dapo_reward("Answer: 41", "42")["score"] == -1.0
    assert rm_hub.f1_score("the cat sat", "cat sat down")[0] == pytest.approx(0.8)
    assert rm_hub.gpqa_reward("The answer is (C).", "C") == 1.0
    assert rm_hub.ifbench_reward("all lower", None, {"instructions": [{"id": "lowercase"}, {"id": "no_comma"}]}) == 1.0
    assert rm_hub.rule_based_reward("boxed_math", r"\boxed{7}", "7") == 1


def test_data_source_buffer_and_resume(tmp_path):
    path = tmp_path / "d.jsonl"
    with open(path, "w") as f:
        for i in range(10):
            f.write(json.dumps({"input": [i, i + 1, i + 2], "label": str(i)}) + "\n")
    a = parse_args(["--prompt-data", str(path), "--label-key", "label", "--n-samples-per-prompt", "2",
                    "--rollout-shuffle", "--rollout-batch-size", "4", "--save", str(tmp_path / "ck")])
    ds = RolloutDataSourceWithBuffer(a)
    g1 = ds.get_samples(3)
    assert len(g1) == 3 and all(len(g) == 2 for g in g1)
    ds.add_samples([g1[0]])
    g2 = ds.get_samples(2)
    assert g2[0] is g1[0]
    ds.save(0)
    st = ds.state_dict()
    ds2 = RolloutDataSourceWithBuffer(a)
    a.load = a.save
    ds2.load(0)
    assert ds2.state_dict() == st
    ex = ds.get_samples(20)  # crosses an epoch boundary
    assert ds.epoch_id >= 1 and len(ex) == 20


def test_dynamic_filter():
    a = parse_args([])
    g = [Sample(reward=1.0), Sample(reward=1.0)]
    assert not check_reward_nonzero_std(a, g).keep
    g[1].reward = 0.0
    assert check_reward_nonzero_std(a, g).keep


def test_sglang_flags_reach_the_engine():
    from miles_b200.orchestration.setup import sglang_engine_kwargs

    kw = sglang_engine_kwargs({"mem_fraction_static": "0.7", "max_running_requests": "96",
                               "chunked_prefill_size": "8192", "disable_cuda_graph": None,
                               "context_length": "32768", "num_continuous_decode_steps": "4",
                               "attention_backend": "fa3"})
    assert kw == {"mem_fraction": 0.7, "max_batch": 96, "prefill_tokens": 8192,
                  "use_cuda_graph": False, "context_length": 32768, "steps_per_sync": 4}
    assert sglang_engine_kwargs({"chunked_prefill_size": "-1"}) == {}
