"""Resharding refit (parallel/reshard.py) on gloo CPU ranks: a trainer in one parallel layout
(TP2, or TP1 x PP2) refits engines in another (TP1, TP2); after the refit every engine's
parameters, gathered to full HF tensors, equal the trainer's (exactly in the full-precision
mode, equal to the 128 x 128 block fp8 round trip of the trainer's weights in fp8 mode)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port


def _full(model):
    from miles_b200.checkpoint.hf import to_hf_tensors
    from miles_b200.parallel.tp import tp_gather_for

    return {n: tp_gather_for(model, n, t.detach()).clone() for n, t in to_hf_tensors(model)}


def _rank(rank, world, port, layout, mode, out):
    os.environ["OMP_NUM_THREADS"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.parallel.reshard import ReshardRefit

    cfg = preset("tiny-moe")
    trainers, engines = layout["trainers"], layout["engines"]
    # groups (every rank creates every group, in the same order)
    tgrp = dist.new_group(trainers)
    egrp = dist.new_group(engines)
    kw = dict(device="cpu", dtype=torch.float32)
    if rank in trainers:
        if layout["train"] == "tp2":
            model = Transformer(cfg, seed=3, tp_group=tgrp, **kw)
        elif layout["train"] == "ep2":
            model = Transformer(cfg, seed=3, ep_group=tgrp, **kw)
        else:
            model = Transformer(cfg, seed=3, pp_group=tgrp, **kw)
    else:
        model = Transformer(cfg, seed=99, tp_group=egrp if layout["engine_tp"] > 1 else None, **kw)
    if layout.get("colocated"):
        # every rank holds a trainer model (PP2 stages) and an engine model (TP2)
        eng = Transformer(cfg, seed=99, tp_group=egrp, **kw)
        refit = ReshardRefit(model, eng, trainers, engines, bucket_bytes=1 << 20, mode=mode)
        refit.update(version=5)
        full = _full(eng)
        assert eng.weight_version == 5
        if eng.tp.rank == 0:
            torch.save(full, f"{out}/e{rank}.pt")
        full_t = _full(model)
        if model.pp.stage >= 0:
            torch.save(full_t, f"{out}/t{model.pp.stage}.pt")
        dist.barrier()
        dist.destroy_process_group()
        return
    refit = ReshardRefit(None if rank in engines else model, model if rank in engines else None,
                         trainers, engines, bucket_bytes=1 << 20, mode=mode)
    stats = refit.update(version=5)
    full = _full(model)
    if rank in engines:
        assert model.weight_version == 5
        assert stats["update_weights/bytes"] > 0
        if model.tp is None or model.tp.rank == 0:
            torch.save(full, f"{out}/e{rank}.pt")
    else:
        stage = model.pp.stage if model.pp is not None else 0
        lead = model.tp is None or model.tp.rank == 0
        if lead:  # EP ranks hold different experts: one file each
            torch.save(full, f"{out}/t{stage}_{rank}.pt")
    dist.barrier()
    dist.destroy_process_group()


LAYOUTS = {
    "tp2_to_tp1": dict(train="tp2", trainers=[0, 1], engines=[2], engine_tp=1),
    "pp2_to_tp2": dict(train="pp2", trainers=[0, 1], engines=[2, 3], engine_tp=2),
    # expert-parallel trainer: each EP rank sends its own experts, EP rank 0 the dense tensors
    "ep2_to_tp2": dict(train="ep2", trainers=[0, 1], engines=[2, 3], engine_tp=2),
    # colocated: the same two ranks hold the trainer (PP2) and the engine (TP2)
    "colocated_pp2_to_tp2": dict(train="pp2", trainers=[0, 1], engines=[0, 1], engine_tp=2,
                                 colocated=True),
}


@pytest.mark.timeout(300)
@pytest.mark.parametrize("name,mode", [("tp2_to_tp1", "bf16"), ("pp2_to_tp2", "bf16"), ("tp2_to_tp1", "fp8"),
                                       ("ep2_to_tp2", "bf16"), ("ep2_to_tp2", "fp8"),
                                       ("colocated_pp2_to_tp2", "bf16")])
def test_reshard_refit(tmp_path, name, mode):
    from miles_b200.ops.quant import fp8_block_dequant, fp8_block_quant

    lay = LAYOUTS[name]
    world = len(set(lay["trainers"]) | set(lay["engines"]))
    mp.spawn(_rank, args=(world, free_port(), lay, mode, str(tmp_path)), nprocs=world, join=True)
    trainer = {}
    for f in sorted(os.listdir(tmp_path)):
        if f.startswith("t"):
            trainer.update(torch.load(tmp_path / f))
    engines = [torch.load(tmp_path / f) for f in os.listdir(tmp_path) if f.startswith("e")]
    assert engines
    if lay["train"] == "ep2":  # both EP ranks' experts arrived
        E = 0
        while any(f".mlp.experts.{E}." in n for n in trainer):
            E += 1
        assert all(any(f".mlp.experts.{e}." in n for n in engines[0]) for e in range(E)) and E > 1
    for eng in engines:
        assert set(eng) <= set(trainer) | {"lm_head.weight"}
        for n, t in eng.items():
            ref = trainer[n]
            if mode == "fp8" and ref.dim() == 2 and min(ref.shape) >= 128:
                q, s = fp8_block_quant(ref.to(torch.bfloat16), (128, 128))
                ref = fp8_block_dequant(q, s, (128, 128), dtype=ref.dtype)
            assert torch.equal(t, ref), n
