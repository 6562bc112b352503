"""Rollout engine on a B200: the device-resident decode loop (several steps per CUDA graph,
stop tokens and length limits handled on the device, routed experts recorded into a device
buffer) reproduces the trainer's log-probs bit for bit, and the fixed-address KV arena keeps
the captured decode graphs valid across release / resume (no re-capture, same outputs)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _model():
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = preset("small-moe")
    return cfg, Transformer(cfg, device="cuda", seed=0)


def _reqs(cfg, n, seed=0, stop=()):
    from miles_b200.engine.engine import GenRequest

    rng = np.random.default_rng(seed)
    return [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(5, 90))).tolist(),
                       int(rng.integers(3, 40)), seed=11 + i, rid=i, return_routed_experts=True,
                       stop_token_ids=stop) for i in range(n)]


def test_device_loop_parity_and_r3():
    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.ops import check_device_error
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.ops.logprob import lm_head_logprob

    cfg, m = _model()
    eng = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4, steps_per_sync=8)
    reqs = _reqs(cfg, 13)  # more requests than slots: later ones join the running batch
    outs = eng.generate(reqs)
    assert eng.stats["host_syncs"] < eng.stats["decode_steps"]
    for r, o in zip(reqs, outs):
        assert len(o.tokens) == r.max_new_tokens and o.finish_reason == "length"
        toks = r.prompt + o.tokens
        rec = []
        with torch.no_grad():
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32, device="cuda"),
                                VarlenMeta([0, len(toks)], "cuda"), record_experts=rec)
            sel = torch.arange(len(r.prompt) - 1, len(toks) - 1, device="cuda")
            lp, _ = lm_head_logprob(h.index_select(0, sel), m.lm_head_weight(),
                                    torch.tensor(o.tokens, dtype=torch.int32, device="cuda"), 1.0, 4096)
        assert torch.equal(lp.float().cpu(), torch.tensor(o.logprobs, dtype=torch.float32))
        ex = torch.stack(rec, 1)[: len(toks) - 1].cpu().numpy()
        assert o.routed_experts.shape == ex.shape and (o.routed_experts == ex).all()
    check_device_error()


def test_stop_tokens_on_device():
    from miles_b200.engine.engine import RolloutEngine

    cfg, m = _model()
    eng = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4)
    free = eng.generate(_reqs(cfg, 6, seed=1))
    # stop on the third token each request produced unconstrained: same prefix, then "stop"
    from miles_b200.engine.engine import GenRequest

    reqs = [GenRequest(r.prompt, r.max_new_tokens, seed=r.seed, rid=r.rid, stop_token_ids=(o.tokens[2],))
            for r, o in zip(_reqs(cfg, 6, seed=1), free) if len(o.tokens) > 3]
    outs = eng.generate(reqs)
    for r, o in zip(reqs, outs):
        ref = next(f for f in free if f.rid == r.rid).tokens
        k = ref.index(r.stop_token_ids[0])
        assert o.tokens == ref[:k + 1] and o.finish_reason == "stop"


def test_graphs_survive_release_resume():
    from miles_b200.engine.engine import RolloutEngine

    cfg, m = _model()
    eng = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4)
    a = eng.generate(_reqs(cfg, 8, seed=2))
    assert eng.arena is not None
    graphs = dict(eng.graphs)
    eng.release_memory()
    x = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")  # other work reuses the memory
    x.fill_(0xFF)
    del x
    b = eng.generate(_reqs(cfg, 8, seed=2))
    assert all(eng.graphs[k] is graphs[k] for k in graphs)  # nothing re-captured
    assert [o.tokens for o in a] == [o.tokens for o in b]
    assert [o.logprobs for o in a] == [o.logprobs for o in b]
