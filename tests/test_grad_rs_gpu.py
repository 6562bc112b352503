"""Fused gradient reduce-scatter over peer memory (csrc/symm.cu grad_rs_kernel,
parallel/symm.py PeerGradBuffer) against a plain fp32 PyTorch reference.

One GPU: W ranks are emulated as W local buffers passed as the "peer" pointers (the kernel only
loads from them; no rank waits on another), each emulated rank reducing its own shard in place;
and a one-rank PeerGradBuffer. Two GPUs (skipped with fewer): FlatAdam steps with the fused
reduce-scatter equal the NCCL ones bitwise (a sum of two bf16 values rounded once is the same
whatever the algorithm)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,n", [(4, 4096 * 8), (8, 8 * 1000), (2, 8 * 37 * 256 + 64)])
def test_grad_rs_emulated_ranks(world, n):
    from miles_b200.ops._lib import lib

    torch.manual_seed(world)
    shard = n // world // 8 * 8
    bufs = [torch.randn(n, device="cuda").to(torch.bfloat16) for _ in range(world)]
    ref = torch.stack([b.float() for b in bufs]).sum(0)
    partial = torch.zeros(592, device="cuda")
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    scale = 0.5
    for r in range(world):
        lo = r * shard
        sq = torch.full((1,), -1.0, device="cuda")
        rc = lib().grad_rs([b.data_ptr() for b in bufs], lo, shard, scale, bufs[r][lo:lo + shard],
                           partial, counter, sq)
        assert rc == 0
        torch.cuda.synchronize()
        want = (ref[lo:lo + shard] * scale).to(torch.bfloat16)
        assert torch.equal(bufs[r][lo:lo + shard], want)
        want_sq = want.float().pow(2).sum().item()
        assert abs(sq.item() - want_sq) <= 1e-5 * want_sq
        assert counter.item() == 0


def test_peer_grad_buffer_one_rank():
    created = not dist.is_initialized()
    if created:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    try:
        from miles_b200.parallel.symm import PeerGradBuffer

        pg = PeerGradBuffer(8 * 5000, dist.group.WORLD, torch.device("cuda", 0))
        x = torch.randn(8 * 5000, device="cuda").to(torch.bfloat16)
        pg.tensor.copy_(x)
        sq = torch.zeros(1, device="cuda")
        for _ in range(3):  # the completion counter resets itself
            pg.reduce_scatter(0, x.numel(), sq)
        torch.cuda.synchronize()
        assert torch.equal(pg.tensor, x)
        assert abs(sq.item() - x.float().pow(2).sum().item()) <= 1e-5 * sq.item()
        pg.close()
    finally:
        if created:
            dist.destroy_process_group()


def _two_rank(rank, port, out):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            device_id=torch.device("cuda", rank))
    from miles_b200.parallel.symm import PeerGradBuffer
    from miles_b200.trainer.optimizer import FlatAdam

    n = 8 * 4096
    res = {}
    for mode in ("nccl", "peer"):
        torch.manual_seed(0)
        p = torch.randn(n, device="cuda").to(torch.bfloat16)
        pg = PeerGradBuffer(n, dist.group.WORLD) if mode == "peer" else None
        g = pg.tensor if pg is not None else torch.zeros(n, dtype=torch.bfloat16, device="cuda")
        opt = FlatAdam(p, g, lr=1e-2, placement="device", dp_group=dist.group.WORLD, peer_grads=pg)
        for step in range(3):
            gen = torch.Generator(device="cuda").manual_seed(100 * step + rank)
            g.copy_(torch.randn(n, device="cuda", generator=gen).to(torch.bfloat16))
            opt.step()
        torch.cuda.synchronize()
        res[mode] = (p.float().cpu(), opt.sq.item())
        if pg is not None:
            pg.close()
    if rank == 0:
        torch.save({"equal": torch.equal(res["nccl"][0], res["peer"][0]),
                    "sq": (res["nccl"][1], res["peer"][1])}, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_grad_rs_two_ranks_matches_nccl(tmp_path):
    out = str(tmp_path / "r.pt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_two_rank, args=(free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["equal"], r
