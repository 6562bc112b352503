"""CPU checks of the cross-cutting utilities: env report, memory report, dumper compare,
profiler window, SFT loss masks, SGLang deployment YAML."""
import os

import torch


def test_env_report_and_memory():
    from miles_b200.utils.env_report import collect
    from miles_b200.utils.memory_utils import available_memory

    rep = collect()
    assert rep["torch"] == torch.__version__ and "git" in rep
    assert isinstance(available_memory(), dict)


def test_dumper_roundtrip(tmp_path):
    from miles_b200.utils import dumper

    dumper._STATE.update(enabled=True, dir=str(tmp_path))
    with dumper.phase("train_fwd", step=3):
        dumper.dump("logp", torch.tensor([1.0, 2.0]))
    with dumper.phase("inference", step=3):
        dumper.dump("logp", torch.tensor([1.0, 2.5]))
    dumper._STATE["enabled"] = False
    r = dumper.compare(str(tmp_path / "train_fwd" / "rank0"), str(tmp_path / "inference" / "rank0"))
    (k, v), = r.items()
    assert abs(v["max_abs"] - 0.5) < 1e-6 and not v["equal"]


def test_profiler_window(tmp_path):
    from types import SimpleNamespace

    from miles_b200.utils.profile_utils import TrainProfiler

    args = SimpleNamespace(use_pytorch_profiler=True, profile_target=["train_overall"],
                           profile_step_start=1, profile_step_end=2, tensorboard_dir=str(tmp_path),
                           record_memory_history=False)
    p = TrainProfiler(args)
    for _ in range(3):
        p.start()
        torch.ones(8) @ torch.ones(8)
        p.stop()
        p.step()
    assert os.listdir(tmp_path / "rank0")


def test_deployment_yaml(tmp_path):
    from types import SimpleNamespace

    from miles_b200.rollout.sglang_config import DeploymentConfig

    (tmp_path / "d.yaml").write_text("""
sglang:
  - name: actor
    server_groups:
      - {worker_type: prefill, num_gpus: 2}
      - {worker_type: decode, num_gpus: 2, overrides: {mem_fraction_static: 0.7}}
  - name: ref
    model_path: /ckpt/ref
    engine_groups:
      - {worker_type: placeholder, num_gpus: 1}
      - {worker_type: regular, num_gpus: 1}
""")
    cfg = DeploymentConfig.from_yaml(str(tmp_path / "d.yaml"))
    assert cfg.total_num_gpus == 6 and cfg.has_pd_disaggregation
    args = SimpleNamespace(hf_checkpoint="/ckpt/actor", rollout_num_gpus_per_engine=1)
    engines, notes = cfg.plan(args, list(range(2, 8)))
    assert [e.ranks[0] for e in engines] == [2, 3, 4, 5, 7]
    assert engines[0].update_weights and not engines[-1].update_weights
    assert engines[2].overrides["mem_fraction_static"] == 0.7
    assert any("prefill" in n for n in notes)


class _ToyTok:
    """Chat template: <role> content </s>, generation prompt '<assistant>'."""
    vocab = {"<system>": 1, "<user>": 2, "<assistant>": 3, "</s>": 4}

    def _w(self, w):
        return self.vocab.get(w, 10 + (hash(w) % 1000))

    def apply_chat_template(self, msgs, tokenize=True, add_generation_prompt=False, **kw):
        ids = []
        for m in msgs:
            ids += [self._w(f"<{m['role']}>")] + [self._w(w) for w in m["content"].split()] + [4]
        if add_generation_prompt:
            ids.append(3)
        return ids


def test_sft_loss_mask():
    from miles_b200.rollout.sft_rollout import build_sft_sample
    from miles_b200.utils.mask_utils import multi_turn_loss_mask
    from miles_b200.utils.types import Sample

    msgs = [{"role": "user", "content": "hi there"}, {"role": "assistant", "content": "hello you"},
            {"role": "user", "content": "more"}, {"role": "assistant", "content": "ok"}]
    ids, mask = multi_turn_loss_mask(_ToyTok(), msgs)
    assert len(ids) == len(mask)
    # user(4 tok) | <assistant>(0) hello you </s> (1,1,1) | user(3) | <assistant>(0) ok </s> (1,1)
    assert mask == [0, 0, 0, 0, 0, 1, 1, 1, 0, 0, 0, 0, 1, 1]
    s = build_sft_sample(_ToyTok(), Sample(prompt=msgs, index=0))
    assert s.response_length == 9 and s.loss_mask == mask[5:]


class _FakeClient:
    def __init__(self):
        self.calls = []

    async def generate(self, ids, sp, return_logprob=True, return_routed_experts=False):
        self.calls.append(list(ids))
        out = [500 + len(self.calls), 4]  # one content token + end-of-turn
        return {"output_ids": out, "text": f"r{len(self.calls)}",
                "meta_info": {"output_token_logprobs": [[-0.5, t] for t in out],
                              "finish_reason": {"type": "stop"}}}


def test_session_server_tito():
    from fastapi.testclient import TestClient

    from miles_b200.rollout.session import SessionRegistry, build_session_app

    tok, client = _ToyTok(), _FakeClient()
    reg = SessionRegistry(tok, client)
    app = TestClient(build_session_app(reg))
    sid = app.post("/sessions").json()["session_id"]
    m1 = [{"role": "user", "content": "solve it"}]
    r1 = app.post(f"/sessions/{sid}/v1/chat/completions", json={"messages": m1}).json()
    assert r1["choices"][0]["message"]["content"] == "r1"
    m2 = m1 + [r1["choices"][0]["message"], {"role": "tool", "content": "42"}]
    app.post(f"/sessions/{sid}/v1/chat/completions", json={"messages": m2})
    # second prompt = first checkpoint tokens (as generated) + tool turn + generation prompt
    first = client.calls[0] + [501, 4]
    assert client.calls[1][:len(first)] == first
    assert client.calls[1][len(first):] == [tok._w("<tool>"), tok._w("42"), 4, 3]
    traj = app.get(f"/sessions/{sid}").json()
    mask = traj["loss_mask"]
    assert sum(mask) == 4 and mask[len(first) - 2:len(first)] == [1, 1] and mask[-2:] == [1, 1]
    # retry from the first checkpoint: rolls back one assistant step
    app.post(f"/sessions/{sid}/v1/chat/completions", json={"messages": m2})
    assert app.get(f"/sessions/{sid}").json()["num_turns"] == 2
    s = reg.get(sid).to_sample()
    assert s.response_length == len(s.loss_mask) and s.loss_mask[0] == 1
    assert app.post("/sessions/nope/v1/chat/completions", json={"messages": m1}).status_code == 404


def test_engine_continuous_batching_matches_single_requests():
    """More requests than batch slots with different lengths: requests join the running batch
    as others finish, and every result equals the request generated alone (greedy and seeded
    sampling); the GDN hybrid (per-sequence state rows recycled) included."""
    import os

    os.environ.setdefault("MILES_B200_FORCE_CPU", "1")
    import numpy as np
    import torch

    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    for name in ("tiny", "tiny-gdn"):
        cfg = preset(name)
        m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
        rng = np.random.default_rng(0)
        reqs = [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(3, 30))).tolist(),
                           int(rng.integers(1, 12)), temperature=0.0 if i % 2 else 1.0, seed=i, rid=i)
                for i in range(9)]
        eng = RolloutEngine(m, max_batch=3, num_pages=64, max_pages_per_seq=4, use_cuda_graph=False)
        outs = eng.generate(reqs)
        assert eng.stats["prefills"] > 1  # later requests joined a running batch
        solo = RolloutEngine(m, max_batch=1, num_pages=64, max_pages_per_seq=4, use_cuda_graph=False)
        for r, o in zip(reqs, outs):
            ref = solo.generate([r])[0]
            assert o.tokens == ref.tokens and len(o.tokens) == r.max_new_tokens, (name, r.rid)
            assert np.allclose(o.logprobs, ref.logprobs, atol=1e-5)
