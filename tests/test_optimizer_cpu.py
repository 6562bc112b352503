"""Sharded (ZeRO-1) flat Adam on a 2-rank gloo world equals the unsharded optimizer applied to
the summed gradients."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port


def _init_params(n):
    g = torch.Generator().manual_seed(0)
    return (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)


def _grads(n, rank):
    g = torch.Generator().manual_seed(100 + rank)
    return (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)


def _worker(rank, world, port, n, out_path):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    from miles_b200.trainer.optimizer import FlatAdam

    p = _init_params(n)
    g = _grads(n, rank)
    opt = FlatAdam(p, g, lr=1e-2, placement="device", dp_group=dist.group.WORLD, clip_grad=1.0)
    for _ in range(2):
        opt.g.copy_(_grads(n, rank))
        opt.step()
    if rank == 0:
        torch.save({"p": p.clone(), "norm": float(opt.grad_norm())}, out_path)
    else:
        torch.save({"p": p.clone()}, out_path + ".1")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_sharded_adam_matches_unsharded(tmp_path):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    from miles_b200.trainer.optimizer import FlatAdam

    n, world = 8192 * 2, 2
    out = str(tmp_path / "r0.pt")
    mp.spawn(_worker, args=(world, free_port(), n, out), nprocs=world, join=True)
    r0 = torch.load(out)
    r1 = torch.load(out + ".1")
    assert torch.equal(r0["p"], r1["p"])  # every rank holds the gathered parameters
    # reference: one optimizer over the summed gradient (bf16 sum, as the collective does)
    p = _init_params(n)
    ref = FlatAdam(p, torch.zeros(n, dtype=torch.bfloat16), lr=1e-2, placement="device",
                   clip_grad=1.0)
    for _ in range(2):
        ref.g.copy_(_grads(n, 0) + _grads(n, 1))
        ref.step()
    assert torch.allclose(r0["p"].float(), p.float(), atol=1e-3, rtol=0)
    assert abs(r0["norm"] - float(ref.grad_norm())) < 1e-3 * float(ref.grad_norm()) + 1e-6
