"""On a B200: a decode engine continuing prefill hand-offs produces bitwise the tokens, log-probs
and routing of a single engine; with int4 QAT on, the engine's decode log-probs equal the training
forward's (the expert GEMMs see the same fake-int4 weights)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _reqs(cfg, n=10):
    from miles_b200.engine.engine import GenRequest

    rng = np.random.default_rng(0)
    return [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(5, 90))).tolist(),
                       int(rng.integers(3, 30)), seed=11 + i, rid=i, return_routed_experts=True)
            for i in range(n)]


def _model():
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = preset("small-moe")
    return cfg, Transformer(cfg, device="cuda", seed=0)


def test_prefill_decode_handoff_bitwise():
    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.ops import check_device_error

    cfg, m = _model()
    pre = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4, use_cuda_graph=False)
    hs = pre.prefill_handoffs(_reqs(cfg))
    pre.release_memory(("kv_cache", "cuda_graph"))
    dec = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4)
    outs = dec.generate(hs)
    assert dec.stats["prefills"] == 0
    dec.release_memory(("kv_cache", "cuda_graph"))
    ref = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4).generate(_reqs(cfg))
    for o, e in zip(outs, ref):
        assert o.tokens == e.tokens and o.logprobs == e.logprobs
        assert (o.routed_experts == e.routed_experts).all()
    check_device_error()


def test_int4_qat_rollout_train_parity():
    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.ops import check_device_error
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.ops.logprob import lm_head_logprob

    cfg, m = _model()
    m.enable_int4_qat(128)
    eng = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4)
    reqs = _reqs(cfg, 6)
    outs = eng.generate(reqs)
    for r, o in zip(reqs, outs):
        toks = r.prompt + o.tokens
        with torch.no_grad():
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32, device="cuda"),
                                VarlenMeta([0, len(toks)], "cuda"))
            sel = torch.arange(len(r.prompt) - 1, len(toks) - 1, device="cuda")
            lp, _ = lm_head_logprob(h.index_select(0, sel), m.lm_head_weight(),
                                    torch.tensor(o.tokens, dtype=torch.int32, device="cuda"), 1.0, 4096)
        assert torch.equal(lp.float().cpu(), torch.tensor(o.logprobs, dtype=torch.float32))
    check_device_error()
