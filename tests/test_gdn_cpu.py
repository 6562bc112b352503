"""Gated DeltaNet hybrid (Qwen3-Next-style) on CPU: engine decode through the recurrent-state
cache reproduces the full forward, the recurrence equals a step-by-step reference, training
backpropagates, HF save/load round-trips, and train.py runs a GRPO step."""
import json
import math
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

from miles_b200.models.config import preset  # noqa: E402
from miles_b200.models.transformer import Transformer  # noqa: E402


def test_gdn_decode_matches_full_forward():
    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.ops.attention import VarlenMeta

    cfg = preset("tiny-gdn")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
    assert m.gdn is not None and "layers.0.linear_attn.in_proj_qkvz.weight" in m.params
    assert "layers.3.self_attn.q_proj.weight" in m.params
    eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=8, use_cuda_graph=False)
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (7, 33, 18)]
    outs = eng.generate([GenRequest(p, 6 + i, temperature=0.0, rid=i) for i, p in enumerate(prompts)])
    for p, o in zip(prompts, outs):
        toks = p + o.tokens
        with torch.no_grad():
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32), VarlenMeta([0, len(toks)], "cpu"))
        logits = h.float() @ m.lm_head_weight().float().t()
        assert logits[len(p) - 1:len(toks) - 1].argmax(-1).tolist() == o.tokens
        lp = torch.log_softmax(logits[len(p) - 1:len(toks) - 1], -1)
        ref = lp.gather(1, torch.tensor(o.tokens)[:, None])[:, 0].detach().numpy()
        assert np.abs(ref - np.asarray(o.logprobs)).max() < 1e-4


def test_gdn_recurrence_reference_and_backward():
    from miles_b200.models.gdn import GDN

    cfg = preset("tiny-gdn")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    g = GDN(m)
    T, nv, dk, dv = 9, g.nv, g.dk, g.dv
    torch.manual_seed(0)
    q = F.normalize(torch.randn(T, nv, dk), dim=-1)
    k = F.normalize(torch.randn(T, nv, dk), dim=-1)
    v = torch.randn(T, nv, dv)
    beta = torch.rand(T, nv)
    lg = -torch.rand(T, nv)
    o, S = g._recur(q, k, v, beta, lg, torch.zeros(nv, dk, dv))
    # explicit state-transition form: S_t = a_t (I - b_t k k^T) S_{t-1} + b_t k v^T
    Sr = torch.zeros(nv, dk, dv)
    for t in range(T):
        for h in range(nv):
            a = math.exp(lg[t, h])
            P = torch.eye(dk) - beta[t, h] * torch.outer(k[t, h], k[t, h])
            Sr[h] = P @ (a * Sr[h]) + beta[t, h] * torch.outer(k[t, h], v[t, h])
            assert torch.allclose(o[t, h], (q[t, h] @ Sr[h]) / math.sqrt(dk), atol=1e-5)
    assert torch.allclose(S, Sr, atol=1e-5)
    from miles_b200.ops.attention import VarlenMeta

    m.recompute = False
    toks = torch.randint(0, cfg.vocab_size, (30,), dtype=torch.int32)
    h = m.forward_train(toks, VarlenMeta([0, 11, 30], "cpu"))
    h.pow(2).mean().backward()
    for n in ("layers.0.linear_attn.A_log", "layers.1.linear_attn.conv1d.weight",
              "layers.2.linear_attn.in_proj_qkvz.weight", "layers.3.self_attn.q_proj.weight"):
        assert m.params[n].grad is not None and m.params[n].grad.abs().sum() > 0, n


def test_gdn_hf_roundtrip_and_grpo_step(tmp_path):
    from miles_b200.checkpoint.hf import load_hf, save_hf

    cfg = preset("tiny-gdn")
    a = Transformer(cfg, device="cpu", dtype=torch.float32, seed=3)
    save_hf(a, str(tmp_path / "hf"))
    b = Transformer(cfg, device="cpu", dtype=torch.float32, seed=4)
    load_hf(b, str(tmp_path / "hf"))
    assert torch.equal(a.flat, b.flat)
    sys.path.insert(0, ROOT)
    rng = np.random.default_rng(0)
    with open(tmp_path / "d.jsonl", "w") as f:
        for _ in range(4):
            f.write(json.dumps({"input": rng.integers(0, 4096, 24).tolist(), "label": "1"}) + "\n")
    import train as T
    from miles_b200.rollout.default import GenerateState
    from miles_b200.utils.arguments import parse_args

    GenerateState._inst = None
    args = parse_args(["--model-name", "tiny-gdn", "--prompt-data", str(tmp_path / "d.jsonl"),
                       "--label-key", "label", "--rollout-batch-size", "2", "--n-samples-per-prompt", "2",
                       "--rollout-max-response-len", "8", "--rm-type", "random", "--num-rollout", "1",
                       "--lr", "1e-3", "--max-tokens-per-gpu", "1024", "--actor-num-gpus-per-node", "1"])
    hist = T.train(args)
    assert len(hist) == 1 and np.isfinite(hist[0]["train/pg_loss"])
    assert hist[0]["train/train_rollout_logprob_abs_diff"] < 1e-4


def test_gdn_chunked_equals_recurrence():
    from miles_b200.models.gdn import GDN

    cfg = preset("tiny-gdn")
    g = GDN(Transformer(cfg, device="cpu", dtype=torch.float32, seed=1))
    torch.manual_seed(1)
    for T in (1, 5, 64, 150):
        q = F.normalize(torch.randn(T, g.nv, g.dk), dim=-1)
        k = F.normalize(torch.randn(T, g.nv, g.dk), dim=-1)
        v = torch.randn(T, g.nv, g.dv)
        beta = torch.rand(T, g.nv)
        lg = -torch.rand(T, g.nv) * 0.5
        S0 = torch.randn(g.nv, g.dk, g.dv) * 0.1
        o1, S1 = g._recur(q, k, v, beta, lg, S0)
        o2, S2 = g._recur_chunked(q, k, v, beta, lg, S0, chunk=64)
        assert torch.allclose(o1, o2, atol=2e-5, rtol=1e-4), (T, (o1 - o2).abs().max())
        assert torch.allclose(S1, S2, atol=2e-5, rtol=1e-4)
