"""DeepSeek-style MLA + MoE model on CPU: training forward/backward, prefill/decode through the
compressed latent cache equals the full forward, and one GRPO step through train.py."""
import os

import numpy as np
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")

from miles_b200.models.config import preset  # noqa: E402
from miles_b200.models.transformer import Transformer  # noqa: E402


def test_mla_decode_matches_full_forward():
    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.ops.attention import VarlenMeta

    cfg = preset("tiny-mla")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
    assert "layers.0.self_attn.kv_b_proj.weight" in m.params and m.mla is not None
    eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=8, use_cuda_graph=False)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (5, 70)]
    outs = eng.generate([GenRequest(p, 6, temperature=0.0, rid=i) for i, p in enumerate(prompts)])
    for p, o in zip(prompts, outs):
        toks = p + o.tokens
        with torch.no_grad():
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32), VarlenMeta([0, len(toks)], "cpu"))
        logits = h.float() @ m.lm_head_weight().float().t()
        greedy = logits[len(p) - 1:len(toks) - 1].argmax(-1).tolist()
        assert greedy == o.tokens
        lp = torch.log_softmax(logits[len(p) - 1:len(toks) - 1], -1)
        ref = lp.gather(1, torch.tensor(o.tokens)[:, None])[:, 0].detach().numpy()
        assert np.abs(ref - np.asarray(o.logprobs)).max() < 1e-3


def test_mla_backward():
    from miles_b200.ops.attention import VarlenMeta

    cfg = preset("tiny-mla")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
    m.recompute = False
    toks = torch.randint(0, cfg.vocab_size, (40,), dtype=torch.int32)
    h = m.forward_train(toks, VarlenMeta([0, 17, 40], "cpu"))
    h.float().pow(2).mean().backward()
    g = m.params["layers.0.self_attn.kv_b_proj.weight"].grad
    assert g is not None and torch.isfinite(g).all() and g.abs().sum() > 0


def test_mla_grpo_step(tmp_path, monkeypatch):
    import json
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    rng = np.random.default_rng(0)
    with open(tmp_path / "d.jsonl", "w") as f:
        for _ in range(4):
            f.write(json.dumps({"input": rng.integers(0, 4096, 32).tolist(), "label": "1"}) + "\n")
    import train as T
    from miles_b200.rollout.default import GenerateState
    from miles_b200.utils.arguments import parse_args

    GenerateState._inst = None
    args = parse_args(["--model-name", "tiny-mla", "--prompt-data", str(tmp_path / "d.jsonl"),
                       "--label-key", "label", "--rollout-batch-size", "2", "--n-samples-per-prompt", "2",
                       "--rollout-max-response-len", "8", "--rm-type", "random", "--num-rollout", "1",
                       "--lr", "1e-3", "--max-tokens-per-gpu", "1024", "--actor-num-gpus-per-node", "1",
                       "--use-tis", "--use-rollout-routing-replay"])
    hist = T.train(args)
    assert len(hist) == 1 and np.isfinite(hist[0]["train/pg_loss"])


def test_dsa_decode_matches_full_forward_and_sparsifies():
    """DSA (MLA + lightning indexer top-k): engine decode through the latent + indexer-key cache
    reproduces the full forward, and the top-k selection changes the output once sequences are
    longer than index_topk."""
    import dataclasses

    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.ops.attention import VarlenMeta

    cfg = preset("tiny-dsa")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
    assert "layers.0.self_attn.indexer.wq_b.weight" in m.params
    eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=8, use_cuda_graph=False)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (9, 70)]
    outs = eng.generate([GenRequest(p, 6, temperature=0.0, rid=i) for i, p in enumerate(prompts)])
    for p, o in zip(prompts, outs):
        toks = p + o.tokens
        with torch.no_grad():
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32), VarlenMeta([0, len(toks)], "cpu"))
        logits = h.float() @ m.lm_head_weight().float().t()
        assert logits[len(p) - 1:len(toks) - 1].argmax(-1).tolist() == o.tokens
        lp = torch.log_softmax(logits[len(p) - 1:len(toks) - 1], -1)
        ref = lp.gather(1, torch.tensor(o.tokens)[:, None])[:, 0].detach().numpy()
        assert np.abs(ref - np.asarray(o.logprobs)).max() < 1e-3
    # dense attention (top-k >= length) gives a different function on the long sequence
    dense = Transformer(dataclasses.replace(cfg, index_topk=4096), device="cpu", dtype=torch.float32,
                        materialize=False)
    dense.flat.copy_(m.flat)
    t = torch.tensor(prompts[1], dtype=torch.int32)
    with torch.no_grad():
        a = m.forward_train(t, VarlenMeta([0, len(t)], "cpu"))
        b = dense.forward_train(t, VarlenMeta([0, len(t)], "cpu"))
    assert torch.allclose(a[:16], b[:16], atol=1e-5)       # first 16 queries see <= 16 keys
    assert (a[20:] - b[20:]).abs().max() > 1e-4
