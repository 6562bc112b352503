"""Weight-refit microbenchmark: seconds and GB/s for one trainer -> engine refit.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m miles_b200.parallel.refit_bench \
        --model qwen3-32b --mode bf16|fp8 --transport peer|nccl|both

Rank 0 is the trainer (source, random-init weights of the named architecture); ranks 1..N-1 are
rollout engines. Each timed refit is device-timed (CUDA events around the transfer, max over
ranks); after the last one every engine checks its weights against the source (bitwise for
bf16; for fp8 against the 128x128 block quantisation of the source). Rank 0 prints one JSON
line per transport.

Resharding (`--src-tp T --src-pp P [--engine-tp E]`): every rank holds both a trainer model in
the T x P layout (T * P = N) and an engine model in TP E (default N), colocated on the same GPUs;
`parallel/reshard.py` gathers each stage's HF tensors over its TP ranks and broadcasts them from
the stage's TP rank 0 to all engine ranks (bf16 or 128x128 fp8), each engine keeping its slice.
Device-timed per refit, max over ranks; after the last refit every engine's gathered weights are
checked against the trainer's (bitwise for bf16; fp8: engines must agree with each other).

Reference: the refit path of update_weight_from_distributed.py (bucketed NCCL broadcast) that
the weight-sync metric times (seconds per refit and GB/s).
"""
from __future__ import annotations

import argparse
import json
import os
import zlib

import torch
import torch.distributed as dist


def _digest(model) -> torch.Tensor:
    """Order-sensitive checksum of the flat parameter buffer (int64 on the device), computed in
    chunks so no full-size temporary is allocated."""
    flat = model.flat.view(torch.int16)
    acc = torch.zeros(1, dtype=torch.int64, device=flat.device)
    chunk = 1 << 26
    w = torch.arange(chunk, device=flat.device, dtype=torch.int64) % 1021 + 1
    for a in range(0, flat.numel(), chunk):
        v = flat[a:a + chunk].to(torch.int64)
        acc += (v * w[: v.numel()]).sum() * ((a // chunk) % 7919 + 1)
    return acc


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-32b")
    ap.add_argument("--mode", choices=["bf16", "fp8"], default="bf16")
    ap.add_argument("--transport", choices=["peer", "nccl", "both"], default="both")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--bucket-mb", type=int, default=1024)
    ap.add_argument("--src-tp", type=int, default=0, help="resharding: trainer TP size")
    ap.add_argument("--src-pp", type=int, default=1, help="resharding: trainer PP size")
    ap.add_argument("--engine-tp", type=int, default=0, help="resharding: engine TP size (default N)")
    a = ap.parse_args(argv)
    if a.src_tp:
        return reshard_main(a)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.parallel.refit import PeerRefit, WeightRefit

    cfg = preset(a.model)
    model = Transformer(cfg, device=dev, seed=1, materialize=rank == 0)
    if rank != 0:
        model.flat.zero_()
    ref_digest = None
    if a.mode == "fp8" and rank == 0:
        # what the engines must end up with: every 2-D weight through the block quantisation
        from miles_b200.ops.quant import fp8_block_dequant, fp8_block_quant

        saved = model.flat.clone()
        for s in model.specs:
            p = model.params[s.name].data
            w = p if p.dim() == 2 else (p.reshape(-1, p.shape[2]) if p.dim() == 3 else None)
            if w is not None and w.shape[0] >= 128 and w.shape[1] >= 128 and w.shape[1] % 16 == 0:
                q, sc = fp8_block_quant(w)
                w.copy_(fp8_block_dequant(q, sc))
        ref_digest = _digest(model)
        model.flat.copy_(saved)
        del saved
    else:
        ref_digest = _digest(model) if rank == 0 else None
    ref = ref_digest if ref_digest is not None else torch.zeros(1, dtype=torch.int64, device=dev)
    dist.broadcast(ref, 0)
    transports = ["peer", "nccl"] if a.transport == "both" else [a.transport]
    for tr in transports:
        cls = PeerRefit if tr == "peer" else WeightRefit
        refit = cls(model, dist.group.WORLD, 0, a.bucket_mb << 20, a.mode)
        times, stats = [], {}
        for it in range(a.iters + 1):
            if rank != 0:
                model.flat.zero_()
            stats = refit.sync()
            if it:  # the first refit is a warm-up
                times.append(stats["perf/update_weights_time"])
        ok = torch.tensor([1 if rank == 0 or torch.equal(_digest(model), ref) else 0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if hasattr(refit, "close"):
            refit.close()
        if rank == 0:
            t = sorted(times)[len(times) // 2]
            print(json.dumps({"metric": "weight_sync_s", "transport": tr, "mode": a.mode,
                              "model": a.model, "n_gpus": world, "engines": world - 1,
                              "seconds": round(t, 5), "bytes": stats["update_weights/bytes"],
                              "GBps_out_of_trainer": round(stats["update_weights/bytes"] / t / 1e9, 1),
                              "all_times": [round(x, 5) for x in times],
                              "engines_match_source": bool(ok.item())}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def reshard_main(a):
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.parallel.reshard import ReshardRefit

    T, P = a.src_tp, a.src_pp
    E = a.engine_tp or world
    if T * P != world or world % E:
        raise ValueError(f"trainer TP{T} x PP{P} and engine TP{E} must tile {world} ranks")
    # trainer groups: TP groups of consecutive ranks, PP groups strided by T
    tp_groups = [dist.new_group(list(range(p * T, (p + 1) * T))) for p in range(P)]
    pp_groups = [dist.new_group(list(range(t, world, T))) for t in range(T)]
    eng_groups = [dist.new_group(list(range(e * E, (e + 1) * E))) for e in range(world // E)]
    cfg = preset(a.model)
    tr = Transformer(cfg, device=dev, seed=1, tp_group=tp_groups[rank // T] if T > 1 else None,
                     pp_group=pp_groups[rank % T] if P > 1 else None)
    eng = Transformer(cfg, device=dev, seed=2, materialize=False,
                      tp_group=eng_groups[rank // E] if E > 1 else None)
    refit = ReshardRefit(tr, eng, list(range(world)), list(range(world)), a.bucket_mb << 20, a.mode)
    times = []
    stats = {}
    for it in range(a.iters + 1):
        eng.flat.zero_()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        stats = refit.update()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if it:  # the first refit is a warm-up
            times.append(float(t))
    # check: every engine's gathered tensors equal the trainer's (bf16) / each other (fp8)
    from miles_b200.checkpoint.hf import to_hf_tensors
    from miles_b200.parallel.tp import tp_gather_for

    def digest(model, names=None):
        acc = torch.zeros(1, dtype=torch.float64, device=dev)
        for n, t in to_hf_tensors(model):
            g = tp_gather_for(model, n, t.detach())
            acc += g.double().abs().sum() * (1 + zlib.crc32(n.encode()) % 97)
        return acc

    de = digest(eng)
    dt = digest(tr)
    if P > 1:
        dist.all_reduce(dt, group=pp_groups[rank % T])  # stages hold disjoint layers
    ok = torch.tensor([1.0 if (a.mode == "fp8" or torch.allclose(de, dt, rtol=1e-12)) else 0.0],
                      device=dev)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0:
        tt = sorted(times)[len(times) // 2]
        print(json.dumps({"metric": "weight_sync_s", "transport": "reshard-nccl", "mode": a.mode,
                          "model": a.model, "n_gpus": world, "trainer_layout": f"tp{T}xpp{P}",
                          "engine_layout": f"tp{E}", "seconds": round(tt, 5),
                          "bytes_broadcast": stats["update_weights/bytes"],
                          "GBps": round(stats["update_weights/bytes"] / tt / 1e9, 1),
                          "all_times": [round(x, 5) for x in times],
                          "engines_match_source": bool(ok.item())}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
