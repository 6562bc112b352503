"""Prefill / decode disaggregation on two gloo ranks: rank 0 prefills (prompt K/V rows, first
token, routing) and sends the hand-offs, rank 1 continues them; the results equal a single
engine's generation of the same requests."""
import os

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port


def _reqs(cfg):
    from miles_b200.engine.engine import GenRequest

    rng = np.random.default_rng(0)
    return [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(8, 70))).tolist(),
                       int(rng.integers(5, 30)), seed=3 + i, rid=i, return_routed_experts=True)
            for i in range(7)]


def _rank(rank, port, out):
    os.environ["OMP_NUM_THREADS"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    from miles_b200.engine.engine import RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.rollout.pd import recv_handoffs, send_handoffs

    cfg = preset("tiny-moe")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
    if rank == 0:
        eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=4, use_cuda_graph=False)
        hs = eng.prefill_handoffs(_reqs(cfg))
        assert len(hs) == 7 and eng.free_pages and len(eng.free_pages) == 63
        send_handoffs(hs, 1)
    else:
        hs = recv_handoffs(0, "cpu")
        eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=4, use_cuda_graph=False)
        outs = eng.generate(hs)
        assert eng.stats["prefills"] == 0  # nothing recomputed
        ref = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=4,
                            use_cuda_graph=False).generate(_reqs(cfg))
        torch.save({"outs": outs, "ref": ref}, out)
    dist.barrier()
    dist.destroy_process_group()


def test_prefill_decode_handoff(tmp_path):
    out = str(tmp_path / "pd.pt")
    mp.spawn(_rank, args=(free_port(), out), nprocs=2, join=True)
    r = torch.load(out, weights_only=False)
    for o, e in zip(r["outs"], r["ref"]):
        assert o.rid == e.rid and o.tokens == e.tokens and len(o.tokens) > 0
        np.testing.assert_allclose(o.logprobs, e.logprobs, rtol=0, atol=1e-4)
        assert o.routed_experts.shape == e.routed_experts.shape
        assert (o.routed_experts == e.routed_experts).all()
