"""fp8 broadcast refit into an engine that serves block fp8: the engine's e4m3 copies receive the
trainer's quantised values and scales as they are (no re-quantisation), and the copies count as
current for the new weight version."""
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port


def _rank(rank, port, out):
    os.environ["OMP_NUM_THREADS"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.quant import fp8_block_quant
    from miles_b200.parallel.refit import WeightRefit

    cfg = preset("tiny-moe")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1 if rank == 0 else 2)
    if rank == 1:
        m.enable_fp8()
    else:
        m.weight_version = 7
    WeightRefit(m, dist.group.WORLD, 0, mode="fp8").sync()
    if rank == 0:
        ref = {}
        for n in ("layers.0.mlp.experts.w1", "layers.1.self_attn.qkv_proj.weight"):
            p = m.params[n].data
            q, s = fp8_block_quant(p.reshape(-1, p.shape[-1]))
            ref[n] = (q.view(torch.uint8).clone(), s.float().clone())
        torch.save(ref, out + ".ref")
    else:
        got = {n: (m.fp8[n].q.clone(), m.fp8[n].s.clone()) for n in
               ("layers.0.mlp.experts.w1", "layers.1.self_attn.qkv_proj.weight")}
        torch.save({"got": got, "ver": m.weight_version, "fp8ver": m._fp8_version}, out)
        m.disable_fp8()
    dist.barrier()
    dist.destroy_process_group()


def test_fp8_refit_fills_engine_copies(tmp_path):
    out = str(tmp_path / "r.pt")
    mp.spawn(_rank, args=(free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    ref = torch.load(out + ".ref")
    assert r["ver"] == 7 and r["fp8ver"] == 7
    for n, (q, s) in ref.items():
        assert torch.equal(r["got"][n][0], q) and torch.equal(r["got"][n][1], s), n
