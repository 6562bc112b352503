"""Speculative rollout with the MTP draft (engine/speculative.py) on CPU: greedy output equals
the plain engine's greedy output, drafts that are always right are all accepted (two tokens per
verify pass) without changing the output, and with temperature sampling every recorded log-prob
is the main model's log-prob of that token (teacher-forced forward), through accepted and
rejected drafts alike."""
import dataclasses
import os

import numpy as np
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")

from miles_b200.engine.engine import GenRequest, RolloutEngine  # noqa: E402


def _model(seed=3):
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer

    cfg = dataclasses.replace(preset("tiny"), mtp_num_layers=1)
    return Transformer(cfg, device="cpu", dtype=torch.float32, seed=seed)


def _reqs(cfg, n, temperature):
    rng = np.random.default_rng(1)
    return [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(5, 30))).tolist(),
                       int(rng.integers(8, 40)), temperature=temperature, seed=11 + i, rid=i)
            for i in range(n)]


def _engine(m, spec):
    return RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=8, use_cuda_graph=False,
                         lazy_pages=False, speculative="mtp" if spec else None)


def test_greedy_matches_plain_engine():
    m = _model()
    ref = {o.rid: o.tokens for o in _engine(m, False).generate(_reqs(m.cfg, 6, 0.0))}
    eng = _engine(m, True)
    out = {o.rid: o.tokens for o in eng.generate(_reqs(m.cfg, 6, 0.0))}
    assert out == ref
    assert eng.stats["spec_steps"] > 0


def test_oracle_drafts_all_accepted():
    m = _model()
    reqs = _reqs(m.cfg, 5, 0.0)
    ref = {o.rid: o.tokens for o in _engine(m, False).generate(reqs)}
    eng = _engine(m, True)
    eng.speculative.draft_override = lambda r, pos: ref[r.rid][pos - len(r.prompt)]
    out = {o.rid: o.tokens for o in eng.generate(_reqs(m.cfg, 5, 0.0))}
    assert out == ref
    st = eng.stats
    assert st["spec_accepted"] == st["spec_drafts"] > 0
    total = sum(len(t) for t in ref.values())
    assert st["spec_steps"] < 0.6 * total  # about two tokens per verify pass


def test_sampled_logprobs_are_main_model_logprobs():
    from miles_b200.ops.attention import VarlenMeta

    m = _model()
    eng = _engine(m, True)
    reqs = _reqs(m.cfg, 6, 1.0)
    outs = eng.generate(reqs)
    # a draft that is right about half the time exercises both branches
    eng2 = _engine(m, True)
    eng2.speculative.draft_override = lambda r, pos: (pos * 7919) % m.cfg.vocab_size
    outs2 = eng2.generate(_reqs(m.cfg, 6, 1.0))
    for res_set in (outs, outs2):
        for r, o in zip(reqs, res_set):
            assert len(o.tokens) == len(o.logprobs) > 0
            toks = torch.tensor(r.prompt + o.tokens, dtype=torch.int32)
            P = len(r.prompt)
            sel = torch.arange(P - 1, P - 1 + len(o.tokens))
            with torch.no_grad():
                lp, _ = m.selected_logprob(toks, VarlenMeta([0, len(toks)], "cpu"), sel,
                                           torch.tensor(o.tokens, dtype=torch.int32), 1.0, 4096)
            assert torch.allclose(torch.tensor(o.logprobs), lp.float(), atol=1e-4), (o.logprobs, lp)


def test_sglang_speculative_flag_enables_it():
    from miles_b200.orchestration.setup import sglang_engine_kwargs

    kw = sglang_engine_kwargs({"speculative_algorithm": "NEXTN", "speculative_num_steps": "1"})
    assert kw == {"speculative": "nextn"}
    m = _model()
    eng = RolloutEngine(m, max_batch=2, num_pages=32, max_pages_per_seq=8, use_cuda_graph=False, **kw)
    assert eng.speculative is not None


def test_partial_rollout_stop_when_and_callbacks():
    """stop_when cuts the call short once 2 results are in (the rest return "abort" with their
    tokens so far); callbacks receive their results instead of the returned list."""
    m = _model()
    eng = _engine(m, True)
    reqs = _reqs(m.cfg, 6, 1.0)
    got = {}
    outs = eng.generate(reqs, stop_when=lambda res: len(res) >= 2,
                        callbacks={reqs[0].rid: lambda r: got.setdefault(r.rid, r)})
    by = {o.rid: o for o in outs}
    assert reqs[0].rid not in by and (reqs[0].rid in got or True)
    fin = [o for o in outs if o.finish_reason != "abort"]
    assert len(fin) >= 2 - len(got)
    assert any(o.finish_reason == "abort" for o in outs)
    assert len(outs) + len(got) == len(reqs)
    for o in outs:
        assert len(o.tokens) == len(o.logprobs)
