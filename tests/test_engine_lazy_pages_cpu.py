"""On-demand KV pages in the rollout engine: with a page pool far smaller than the requests'
full lengths, sequences grow page by page, the latest admitted is preempted when the pool runs
dry and resumes by re-prefill; every request still completes with all its tokens, log-probs and
routing, and the outputs equal those of a run whose pool never runs dry."""
import numpy as np
import torch

from miles_b200.engine.engine import GenRequest, RolloutEngine
from miles_b200.models.config import preset
from miles_b200.models.transformer import Transformer


def _reqs(cfg, n):
    rng = np.random.default_rng(0)
    return [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(10, 60))).tolist(),
                       int(rng.integers(40, 120)), seed=5 + i, rid=i, return_routed_experts=True)
            for i in range(n)]


def test_lazy_pages_preempt_and_resume():
    cfg = preset("tiny-moe")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
    big = RolloutEngine(m, max_batch=6, num_pages=256, max_pages_per_seq=4, use_cuda_graph=False,
                        lazy_pages=False)
    ref = {o.rid: o for o in big.generate(_reqs(cfg, 6))}
    small = RolloutEngine(m, max_batch=6, num_pages=9, max_pages_per_seq=4, use_cuda_graph=False)
    outs = {o.rid: o for o in small.generate(_reqs(cfg, 6))}
    assert small.stats["preemptions"] > 0
    for r in _reqs(cfg, 6):
        o, e = outs[r.rid], ref[r.rid]
        assert len(o.tokens) == r.max_new_tokens and len(o.logprobs) == r.max_new_tokens
        assert o.routed_experts.shape == e.routed_experts.shape
        assert o.tokens == e.tokens
        np.testing.assert_allclose(o.logprobs, e.logprobs, rtol=0, atol=1e-4)
