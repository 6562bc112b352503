"""Sequence-length balancing: Karmarkar-Karp partitions (equal counts for --balance-data,
free counts for --use-dynamic-batch-size micro-batches), the minimum micro-batch count under
a token budget, and the cross-rank redistribution on two gloo ranks."""
import os
import random

import pytest
import torch.multiprocessing as mp

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def test_kk_partitions_cover_and_balance():
    from miles_b200.utils.seqlen_balancing import karmarkar_karp

    rng = random.Random(0)
    L = [rng.randint(100, 8000) for _ in range(64)]
    for k in (2, 4, 8):
        for eq in (False, True):
            parts = karmarkar_karp(L, k, equal_size=eq)
            assert sorted(i for p in parts for i in p) == list(range(64))
            sums = [sum(L[i] for i in p) for p in parts]
            assert max(sums) - min(sums) <= max(L) // 4 + 1
            if eq:
                assert all(len(p) == 64 // k for p in parts)
    # the round-robin split it replaces is far less balanced on sorted input
    srt = sorted(L)
    rr = [sum(srt[i::4]) for i in range(4)]
    kk = [sum(srt[i] for i in p) for p in karmarkar_karp(srt, 4, True)]
    assert max(kk) - min(kk) < max(rr) - min(rr)
    with pytest.raises(ValueError):
        karmarkar_karp(L[:63], 4, equal_size=True)


def test_micro_batch_counts():
    from miles_b200.trainer.actor import ActorConfig, make_micro_batches
    from miles_b200.utils.seqlen_balancing import minimum_num_micro_batches

    L = [900, 800, 700, 300, 200, 100]
    assert minimum_num_micro_batches(L, 1000) == 3
    mbs = make_micro_batches(L, ActorConfig(max_tokens_per_gpu=1000, micro_batching="balanced"))
    assert len(mbs) == 3 and sorted(i for m in mbs for i in m) == list(range(6))
    assert [sum(L[i] for i in m) for m in mbs] == [1000, 1000, 1000]
    fixed = make_micro_batches(L, ActorConfig(micro_batching="fixed", micro_batch_size=4))
    assert fixed == [[0, 1, 2, 3], [4, 5]]


def _rank(rank, port, out):
    import torch.distributed as dist

    from miles_b200.utils.seqlen_balancing import rebalance_over_dp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    # rank 0 holds the four long samples, rank 1 the four short ones
    lens = [4000, 3900, 3800, 3700] if rank == 0 else [10, 20, 30, 40]
    data = {"tokens": [[rank] * n for n in lens], "rewards": [float(n) for n in lens],
            "metrics": {"x": rank}}
    got = rebalance_over_dp(data, dist.group.WORLD)
    out[rank] = (sum(len(t) for t in got["tokens"]), len(got["tokens"]),
                 [len(t) == int(r) for t, r in zip(got["tokens"], got["rewards"])], got["metrics"])
    dist.destroy_process_group()


def test_rebalance_over_two_ranks():
    from tests.conftest import free_port

    out = mp.Manager().dict()
    mp.spawn(_rank, args=(free_port(), out), nprocs=2)
    tot = [out[r][0] for r in range(2)]
    assert abs(tot[0] - tot[1]) < 500 and sum(tot) == 15500
    assert all(out[r][1] == 4 and all(out[r][2]) for r in range(2))
    assert out[0][3] == {"x": 0} and out[1][3] == {"x": 1}
