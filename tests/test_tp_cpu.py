"""Tensor parallelism on CPU (gloo, 2 ranks): a TP2 model loaded from a TP1 model's HF
checkpoint gives the same training forward, the same (gathered) gradients, the same engine
decode, and saves back the same HF tensors; one optimizer step keeps the TP ranks' replicated
parameters identical."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


def _cfg(name):
    """Presets, plus attention variants that run through the separate-q/k/v path: GLM-4.5-like
    (projection biases, half-width rotary, MoE) and Qwen3-Next-like (output gate, quarter-width
    rotary)."""
    import dataclasses

    from miles_b200.models.config import preset

    if name == "tiny-biased":
        return dataclasses.replace(preset("tiny-moe"), attention_bias=True, partial_rotary_factor=0.5)
    if name == "tiny-sandwich":  # GLM-4-like: sandwich norms, biases, half interleaved rotary
        return dataclasses.replace(preset("tiny"), sandwich_norm=True, attention_bias=True,
                                   partial_rotary_factor=0.5, rope_interleave=True)
    if name == "tiny-gated":
        return dataclasses.replace(preset("tiny"), attn_output_gate=True, partial_rotary_factor=0.25)
    return preset(name)


def _run(rank, world, port, preset_name, ckpt, out_dir):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import preset
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.parallel.tp import tp_gather

    cfg = _cfg(preset_name)
    from miles_b200.models.transformer import Transformer

    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=5, tp_group=dist.group.WORLD)
    assert m.tp is not None and m.tp.size == world and m.tp.backend == "torch"
    load_hf(m, ckpt)
    m.recompute = False
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, cfg.vocab_size, (37,), generator=g, dtype=torch.int32)
    meta = VarlenMeta([0, 15, 37], "cpu")
    h = m.forward_train(toks, meta)
    h.pow(2).mean().backward()
    grads = {}
    from miles_b200.checkpoint.hf import to_hf_tensors  # noqa: F401  (names)
    from miles_b200.parallel.tp import tp_partial_param_names

    partial = set(tp_partial_param_names(m))
    for name, p in m.params.items():
        if p.grad is None:
            continue
        gr = p.grad.clone()
        if name in partial:
            dist.all_reduce(gr)
        grads[name] = gr
    # sequence parallel: same forward, same gradients (37 rows: exercises the padding)
    sp = {}
    if True:  # sequence parallel for every family
        for p in m.params.values():
            p.grad = None
        m.sequence_parallel = True
        hs = m.forward_train(toks, meta)
        hs.pow(2).mean().backward()
        sp["h"] = hs.detach()
        partial_sp = set(tp_partial_param_names(m))
        sp["grads"] = {}
        for name, p in m.params.items():
            if p.grad is None:
                continue
            gr = p.grad.clone()
            if name in partial_sp:
                dist.all_reduce(gr)
            sp["grads"][name] = gr
        m.sequence_parallel = False
    # engine decode (prefill + 4 greedy steps)
    from miles_b200.engine.engine import GenRequest, RolloutEngine

    eng = RolloutEngine(m, max_batch=2, num_pages=16, max_pages_per_seq=4, use_cuda_graph=False)
    outs = eng.generate([GenRequest(toks[:9].tolist(), 4, temperature=0.0, rid=0),
                         GenRequest(toks[9:30].tolist(), 4, temperature=0.0, rid=1)])
    save_hf(m, os.path.join(out_dir, "resaved"))
    if rank == 0:
        torch.save({"h": h.detach(), "grads": grads, "sp": sp, "tokens": [o.tokens for o in outs],
                    "lps": [o.logprobs for o in outs]}, os.path.join(out_dir, f"tp{world}.pt"))
    dist.destroy_process_group()


def _single(preset_name, ckpt):
    from miles_b200.checkpoint.hf import save_hf
    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    cfg = _cfg(preset_name)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=11)
    save_hf(m, ckpt)
    m.recompute = False
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, cfg.vocab_size, (37,), generator=g, dtype=torch.int32)
    h = m.forward_train(toks, VarlenMeta([0, 15, 37], "cpu"))
    h.pow(2).mean().backward()
    eng = RolloutEngine(m, max_batch=2, num_pages=16, max_pages_per_seq=4, use_cuda_graph=False)
    outs = eng.generate([GenRequest(toks[:9].tolist(), 4, temperature=0.0, rid=0),
                         GenRequest(toks[9:30].tolist(), 4, temperature=0.0, rid=1)])
    return m, h.detach(), outs


def _rank0_slice(name, full, cfg, t):
    """Rank 0's TP slice of a full (TP1) parameter in the internal fused layout."""
    def halves(x, d):
        a, b = x.chunk(2, d)
        return torch.cat([a.narrow(d, 0, a.shape[d] // t), b.narrow(d, 0, b.shape[d] // t)], d)

    from miles_b200.parallel.tp import _gdn_blocks

    blk = _gdn_blocks(name, cfg)  # Gated DeltaNet: every block split by heads
    if blk is not None:
        d, sizes = blk
        parts, off = [], 0
        for n in sizes:
            parts.append(full.narrow(d, off, n // t))
            off += n
        return torch.cat(parts, d)
    if name.endswith("qkv_proj.weight"):
        D = cfg.head_dim
        q, k, v = full.split([cfg.num_heads * D, cfg.num_kv_heads * D, cfg.num_kv_heads * D], 0)
        return torch.cat([x.narrow(0, 0, x.shape[0] // t) for x in (q, k, v)], 0)
    if name.endswith("gate_up_proj.weight"):
        return halves(full, 0)
    if name.endswith("experts.w1"):
        return halves(full, 1)
    if name.endswith("experts.w2"):
        return full.narrow(2, 0, full.shape[2] // t)
    if name.endswith(("o_proj.weight", "down_proj.weight")):
        return full.narrow(1, 0, full.shape[1] // t)
    if name.endswith(("q_proj.weight", "q_b_proj.weight", "kv_b_proj.weight", "k_proj.weight",
                      "v_proj.weight", "q_proj.bias", "k_proj.bias", "v_proj.bias")):
        return full.narrow(0, 0, full.shape[0] // t)
    return full


@pytest.mark.parametrize("preset_name,port", [("tiny", 29671), ("tiny-moe", 29672), ("tiny-mla", 29673),
                                              ("tiny-dsa", 29674), ("tiny-biased", 29675),
                                              ("tiny-gated", 29676), ("tiny-gdn", 29677),
                                              ("tiny-sandwich", 29678)])
def test_tp2_matches_tp1(tmp_path, preset_name, port):
    from safetensors.torch import load_file

    from miles_b200.parallel.tp import hf_shard_dim

    ckpt = str(tmp_path / "ref")
    m1, h1, outs1 = _single(preset_name, ckpt)
    mp.spawn(_run, args=(2, free_port(), preset_name, ckpt, str(tmp_path)), nprocs=2, join=True)
    r = torch.load(tmp_path / "tp2.pt")
    assert torch.allclose(r["h"], h1, atol=2e-5, rtol=1e-4), (r["h"] - h1).abs().max()
    # gradients: rank 0 holds slice 0 of sharded tensors, full replicated ones
    from miles_b200.checkpoint.hf import to_hf_tensors  # noqa: F401

    cfg = m1.cfg
    assert set(r["grads"]) == {n for n, p in m1.params.items() if p.grad is not None}
    for name, g2 in r["grads"].items():
        g1 = _rank0_slice(name, m1.params[name].grad, cfg, 2)
        assert g1.shape == g2.shape, name
        assert torch.allclose(g2, g1, atol=1e-5, rtol=1e-3), (name, (g2 - g1).abs().max())
    if r["sp"]:
        assert torch.allclose(r["sp"]["h"], h1, atol=2e-5, rtol=1e-4), (r["sp"]["h"] - h1).abs().max()
        assert set(r["sp"]["grads"]) == set(r["grads"])
        for name, g2 in r["sp"]["grads"].items():
            g1 = _rank0_slice(name, m1.params[name].grad, cfg, 2)
            assert torch.allclose(g2, g1, atol=1e-5, rtol=1e-3), ("sp", name, (g2 - g1).abs().max())
    assert r["tokens"] == [o.tokens for o in outs1]
    for a, b in zip(r["lps"], [o.logprobs for o in outs1]):
        assert np.abs(np.asarray(a) - np.asarray(b)).max() < 1e-4
    # HF round trip through the TP2 model: gathered tensors equal the source checkpoint
    import glob

    src = {}
    for f in glob.glob(os.path.join(ckpt, "*.safetensors")):
        src.update(load_file(f))
    back = {}
    for f in glob.glob(os.path.join(str(tmp_path / "resaved"), "*.safetensors")):
        back.update(load_file(f))
    assert set(src) == set(back)
    for k in src:
        assert torch.equal(src[k], back[k]), k
    assert any(hf_shard_dim(k) is not None for k in src)


def _run_vp(rank, world, port, out):
    os.environ["MILES_B200_FORCE_CPU"] = "1"
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.parallel.tp import tp_partial_param_names

    cfg = preset("tiny-moe")  # untied LM head
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=5, tp_group=dist.group.WORLD)
    m.recompute = False
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, cfg.vocab_size, (30,), generator=g, dtype=torch.int32)
    meta = VarlenMeta([0, 12, 30], "cpu")
    sel = torch.arange(3, 28)
    tgt = toks[sel + 1]
    res = {}
    for vp in (False, True):
        m.vocab_parallel_logprob = vp
        for p in m.params.values():
            p.grad = None
        lp, ent = m.selected_logprob(toks, meta, sel, tgt, 1.3, 8)
        (lp.sum() + 0.3 * ent.sum()).backward()
        grads = {}
        partial = set(tp_partial_param_names(m))
        for n, p in m.params.items():
            if p.grad is not None:
                gr = p.grad.clone()
                if n in partial:
                    dist.all_reduce(gr)
                grads[n] = gr
        res[vp] = (lp.detach(), ent.detach(), grads)
    if rank == 0:
        torch.save(res, out)
    dist.destroy_process_group()


def test_vocab_parallel_logprob(tmp_path):
    """TP2 log-probs / entropies with the vocabulary split over the ranks equal the replicated
    LM head's, and so do all gradients (LM head rows all-reduced)."""
    out = str(tmp_path / "vp.pt")
    mp.spawn(_run_vp, args=(2, free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    (lp0, e0, g0), (lp1, e1, g1) = r[False], r[True]
    assert torch.allclose(lp0, lp1, atol=1e-5) and torch.allclose(e0, e1, atol=1e-5)
    assert set(g0) == set(g1)
    for n in g0:
        assert torch.allclose(g0[n], g1[n], atol=1e-5, rtol=1e-4), (n, (g0[n] - g1[n]).abs().max())
