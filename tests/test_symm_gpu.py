"""Symmetric-memory collectives (csrc/symm.cu, parallel/symm.py) and tensor parallelism on
B200s.

One GPU: a one-rank group exercises every kernel (the GEMM epilogue that stores into peer
staging, the rank-ordered reduce, the fused residual + RMSNorm, the device-side epoch across
repeated calls and CUDA-graph replays) against the plain kernels, and a wait that runs out
(a peer flag that nothing sets) reports error 3 and leaves the context usable.
Two GPUs (skipped with fewer): the fused paths equal GEMM + NCCL all-reduce + add_rms_norm
bitwise, and a TP2 model's engine decode log-probs equal its trainer forward's.
"""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from tests.conftest import free_port

pytestmark = pytest.mark.gpu


@pytest.fixture
def one_rank_group():
    """A one-rank process group (torn down afterwards so later tests can create their own)."""
    created = not dist.is_initialized()
    if created:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{free_port()}", rank=0, world_size=1)
    yield dist.group.WORLD
    if created:
        dist.destroy_process_group()


def test_symm_single_rank_kernels(one_rank_group):
    from miles_b200.ops import check_device_error
    from miles_b200.ops import gemm as G
    from miles_b200.ops.norm import add_rms_norm
    from miles_b200.parallel.symm import SymmComm

    g = one_rank_group
    torch.cuda.set_device(0)
    H = 2048
    comm = SymmComm(g, hidden=H, cap_rows=256)
    torch.manual_seed(0)
    for it in range(5):  # crosses both staging parities several times
        M = [1, 64, 200, 256, 37][it]
        a = torch.randn(M, 1536, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(H, 1536, device="cuda", dtype=torch.bfloat16) * 0.03
        res = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
        nw = torch.rand(H, device="cuda", dtype=torch.bfloat16) + 0.5
        ref_lin = G.linear(a, w)
        assert torch.equal(comm.gemm_all_reduce(a, w), ref_lin)
        assert torch.equal(comm.all_reduce(ref_lin), ref_lin)
        y_ref, h_ref = add_rms_norm(ref_lin, res, nw, 1e-6)
        y, h = comm.gemm_all_reduce(a, w, res=res, norm_w=nw, eps=1e-6)
        assert torch.equal(h, h_ref) and torch.equal(y, y_ref)
        y2, h2 = comm.all_reduce_add_norm(ref_lin, res, nw, 1e-6)
        assert torch.equal(h2, h_ref) and torch.equal(y2, y_ref)
    # MN-major weight (column-parallel backward form: dy @ W)
    dy = torch.randn(64, 1536, device="cuda", dtype=torch.bfloat16)
    wt = torch.randn(1536, H, device="cuda", dtype=torch.bfloat16) * 0.03
    assert torch.equal(comm.gemm_all_reduce(dy, wt, w_mn=True), G.matmul_nn(dy, wt))
    # CUDA graph: the epoch lives on the device, replays advance it
    a = torch.randn(64, 1536, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, 1536, device="cuda", dtype=torch.bfloat16) * 0.03
    res = torch.randn(64, H, device="cuda", dtype=torch.bfloat16)
    nw = torch.rand(H, device="cuda", dtype=torch.bfloat16) + 0.5
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        comm.gemm_all_reduce(a, w, res=res, norm_w=nw, eps=1e-6)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yg, hg = comm.gemm_all_reduce(a, w, res=res, norm_w=nw, eps=1e-6)
    y_ref, h_ref = add_rms_norm(G.linear(a, w), res, nw, 1e-6)
    e0 = int(comm.ctl[0])
    for _ in range(3):
        yg.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(yg, y_ref) and torch.equal(hg, h_ref)
    assert int(comm.ctl[0]) == e0 + 3
    check_device_error()
    comm.close()


def test_symm_wait_times_out_with_error_status(one_rank_group):
    """A peer flag that nothing sets: the bounded wait gives up, records code 3, and the
    context stays usable."""
    from miles_b200.ops import _lib
    from miles_b200.ops._lib import DeviceKernelError, check_device_error, err_word
    from miles_b200.parallel.symm import SymmComm

    g = one_rank_group
    torch.cuda.set_device(0)
    comm = SymmComm(g, hidden=256, cap_rows=8)
    check_device_error()
    x = torch.ones(4, 256, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(x)
    # a two-rank call whose second "peer" is this rank's own region: slot / flag 1 never arrive
    flags = [comm.flag_ptrs[0], comm.flag_ptrs[0]]
    stage = [comm.stage_ptrs[0], comm.stage_ptrs[0]]
    _lib.lib().symm_allreduce(flags, stage, comm.my_flags, comm.ctl, comm.my_stage, comm.cap, None, 4, 256,
                              0, 2, None, None, 0.0, out, None, None, int(0.05e9), err_word(x.device))
    torch.cuda.synchronize()
    with pytest.raises(DeviceKernelError):
        check_device_error()
    # context still usable, epoch advanced, the one-rank collective works again
    comm.my_flags.zero_()
    comm.ctl.zero_()
    y = comm.all_reduce(x)
    torch.cuda.synchronize()
    assert torch.equal(y, x)
    check_device_error()
    comm.close()


# ------------------------------------------------------------------ two GPUs
def _two_rank(rank, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            device_id=torch.device("cuda", rank))
    from miles_b200.ops import check_device_error
    from miles_b200.ops import gemm as G
    from miles_b200.ops.norm import add_rms_norm
    from miles_b200.parallel.symm import SymmComm

    H = 2048
    comm = SymmComm(dist.group.WORLD, hidden=H, cap_rows=512)
    res = {}
    torch.manual_seed(100 + rank)
    ok = True
    for M in (1, 64, 512):
        a = torch.randn(M, 1024, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(H, 1024, device="cuda", dtype=torch.bfloat16) * 0.03
        r = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
        dist.broadcast(r, 0)
        nw = torch.rand(H, device="cuda", dtype=torch.bfloat16) + 0.5
        dist.broadcast(nw, 0)
        part = G.linear(a, w)
        ref = part.clone()
        dist.all_reduce(ref)
        ok &= torch.equal(comm.all_reduce(part), ref)
        ok &= torch.equal(comm.gemm_all_reduce(a, w), ref)
        y_ref, h_ref = add_rms_norm(ref, r, nw, 1e-6)
        y, h = comm.gemm_all_reduce(a, w, res=r, norm_w=nw, eps=1e-6)
        ok &= torch.equal(y, y_ref) and torch.equal(h, h_ref)
    # reduce-scatter / all-gather / fused GEMM + reduce-scatter
    x = torch.randn(512, H, device="cuda", dtype=torch.bfloat16)
    ref = x.clone()
    dist.all_reduce(ref)
    ok &= torch.equal(comm.reduce_scatter(x), ref[rank * 256:(rank + 1) * 256])
    parts = [torch.empty(100, H, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    dist.all_gather(parts, x[:100].contiguous())
    ok &= torch.equal(comm.all_gather(x[:100]), torch.cat(parts))
    a = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, 1024, device="cuda", dtype=torch.bfloat16) * 0.03
    ref = G.linear(a, w)
    dist.all_reduce(ref)
    ok &= torch.equal(comm.gemm_reduce_scatter(a, w), ref[rank * 256:(rank + 1) * 256])
    res["rs_ag_ok"] = bool(ok)
    # decode-shaped timing: fused GEMM+AR+norm vs GEMM, NCCL all-reduce, add_rms_norm
    M, K = 64, 2048
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, K, device="cuda", dtype=torch.bfloat16) * 0.03
    r = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
    nw = torch.rand(H, device="cuda", dtype=torch.bfloat16) + 0.5

    def fused():
        return comm.gemm_all_reduce(a, w, res=r, norm_w=nw, eps=1e-6)

    def base():
        p = G.linear(a, w)
        dist.all_reduce(p)
        return add_rms_norm(p, r, nw, 1e-6)

    for name, fn in (("fused", fused), ("nccl", base)):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for _ in range(200):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 200 * 1e3], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name + "_us"] = float(t)
    check_device_error()
    # TP2 model: engine decode log-probs == trainer forward log-probs (bitwise)
    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    cfg = preset("small-moe")
    m = Transformer(cfg, device="cuda", seed=3, tp_group=dist.group.WORLD, tp_cap_rows=1024)
    assert m.tp.backend == "symm"
    eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=8, use_cuda_graph=True)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 70, 33)]
    outs = eng.generate([GenRequest(p, 12, temperature=1.0, rid=i, seed=7 + i)
                         for i, p in enumerate(prompts)])
    from miles_b200.ops.logprob import lm_head_logprob

    diff = 0.0
    with torch.no_grad():
        for p, o in zip(prompts, outs):
            toks = p + o.tokens
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32, device="cuda"),
                                VarlenMeta([0, len(toks)], "cuda"))
            sel = torch.arange(len(p) - 1, len(toks) - 1, device="cuda")
            lp, _ = lm_head_logprob(h.index_select(0, sel), m.lm_head_weight(),
                                    torch.tensor(o.tokens, device="cuda"), 1.0, 4096)
            diff = max(diff, (lp.float().cpu() - torch.tensor(o.logprobs)).abs().max().item())
    res["tp2_logprob_diff"] = diff
    # sequence parallel training forward == TP forward (bitwise), and it backpropagates
    toks = torch.randint(0, cfg.vocab_size, (301,), generator=g).to("cuda", torch.int32)
    meta = VarlenMeta([0, 120, 301], "cuda")
    with torch.no_grad():
        h_tp = m.forward_train(toks, meta)
    m.sequence_parallel = True
    h_sp = m.forward_train(toks, meta)
    res["sp_equal"] = bool(torch.equal(h_sp.detach(), h_tp))
    h_sp.float().pow(2).mean().backward()
    gw = m.params["layers.0.self_attn.o_proj.weight"].grad
    res["sp_grad_finite"] = bool(gw is not None and torch.isfinite(gw.float()).all())
    m.sequence_parallel = False
    # context parallel 2: log-probs bitwise equal to the single-GPU forward
    m_cp = Transformer(cfg, device="cuda", seed=4, cp_group=dist.group.WORLD)
    m_1 = Transformer(cfg, device="cuda", seed=4)
    sel = torch.arange(130, 300, device="cuda")
    tgt = toks[sel + 1]
    with torch.no_grad():
        lp_cp, _ = m_cp.selected_logprob(toks, meta, sel, tgt, 1.0, 4096)
        lp_1, _ = m_1.selected_logprob(toks, meta, sel, tgt, 1.0, 4096)
    res["cp_equal"] = bool(torch.equal(lp_cp, lp_1))
    lp_cp, _ = m_cp.selected_logprob(toks, meta, sel, tgt, 1.0, 4096)
    lp_cp.sum().backward()
    res["cp_grad_finite"] = bool(torch.isfinite(m_cp.params["layers.1.self_attn.qkv_proj.weight"].grad.float()).all())
    del m_cp, m_1
    res["tokens"] = [o.tokens for o in outs]
    check_device_error()
    res["ok"] = bool(ok)
    comm.close()
    if rank == 0:
        torch.save(res, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_symm_two_ranks(tmp_path):
    out = str(tmp_path / "r.pt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_two_rank, args=(free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    print({k: v for k, v in r.items() if k != "tokens"})
    assert r["ok"]
    assert r["tp2_logprob_diff"] == 0.0
    assert r["rs_ag_ok"] and r["sp_equal"] and r["sp_grad_finite"]
    assert r["cp_equal"] and r["cp_grad_finite"]


def _two_rank_refit(rank, port, out):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            device_id=torch.device("cuda", rank))
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops import check_device_error
    from miles_b200.parallel.refit import PeerRefit, WeightRefit

    cfg = preset("small-moe")
    m = Transformer(cfg, device="cuda", seed=9, materialize=rank == 0)
    res = {}
    for mode in ("bf16", "fp8"):
        got = {}
        for cls in (WeightRefit, PeerRefit):
            if rank == 1:
                m.flat.zero_()
            r = cls(m, dist.group.WORLD, 0, 4 << 20, mode)  # small buckets: several rounds
            st = r.sync()
            got[cls.__name__] = m.flat.clone()
            if hasattr(r, "close"):
                r.close()
            res[f"{mode}_{cls.__name__}_GBps"] = st["update_weights/GBps"]
        if rank == 1:
            res[f"{mode}_equal"] = bool(torch.equal(got["WeightRefit"], got["PeerRefit"]))
            res[f"{mode}_nonzero"] = bool(got["PeerRefit"].abs().sum() > 0)
    check_device_error()
    if rank == 1:
        torch.save(res, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_refit_matches_nccl_refit(tmp_path):
    out = str(tmp_path / "refit.pt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_two_rank_refit, args=(free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    print(r)
    assert r["bf16_equal"] and r["fp8_equal"] and r["bf16_nonzero"]


def _two_rank_ep(rank, port, out, world=2):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops import check_device_error
    from miles_b200.ops.attention import VarlenMeta

    cfg = preset("small-moe")
    m = Transformer(cfg, device="cuda", seed=21 + rank, ep_group=dist.group.WORLD, ep_cap_tokens=1024)
    assert m.ep is not None and m.ep.transport == "peer"
    g = torch.Generator().manual_seed(5 + rank)  # different tokens per rank
    toks = torch.randint(0, cfg.vocab_size, (333,), generator=g).to("cuda", torch.int32)
    meta = VarlenMeta([0, 100, 333], "cuda")
    res = {}
    outs, grads = {}, {}
    for tr in ("peer", "nccl"):
        m.ep.transport = tr
        for p in m.params.values():
            p.grad = None
        h = m.forward_train(toks, meta)
        h.float().pow(2).mean().backward()
        outs[tr] = h.detach().clone()
        grads[tr] = {n: p.grad.clone() for n, p in m.params.items() if p.grad is not None}
    res["fwd_equal"] = bool(torch.equal(outs["peer"], outs["nccl"]))
    res["grad_equal"] = all(torch.equal(grads["peer"][n], grads["nccl"][n]) for n in grads["nccl"])
    res["grad_names"] = sorted(grads["nccl"])
    # decode-sized forward without autograd
    with torch.no_grad():
        hs = {}
        for tr in ("peer", "nccl"):
            m.ep.transport = tr
            hs[tr] = m.forward_train(toks[:40], VarlenMeta([0, 40], "cuda"))
        res["nograd_equal"] = bool(torch.equal(hs["peer"], hs["nccl"]))
    check_device_error()
    if rank == 0:
        torch.save(res, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_peer_transport_matches_nccl(tmp_path):
    out = str(tmp_path / "ep.pt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_two_rank_ep, args=(free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    print(r)
    assert r["fwd_equal"] and r["grad_equal"] and r["nograd_equal"]


@pytest.mark.parametrize("world", [4, 8])
def test_ep_peer_transport_matches_nccl_n_ranks(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = str(tmp_path / "ep.pt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_two_rank_ep, args=(free_port(), out, world), nprocs=world, join=True)
    r = torch.load(out)
    assert r["fwd_equal"] and r["grad_equal"] and r["nograd_equal"]


def _n_rank_collectives(rank, port, out, world):
    """Symmetric collectives at `world` ranks against a rank-ordered reference: every rank's
    part gathered with NCCL and summed in rank order in fp32, rounded once (the symmetric
    kernels' arithmetic; NCCL's own all-reduce order differs above two ranks)."""
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, device_id=torch.device("cuda", rank))
    from miles_b200.ops import check_device_error
    from miles_b200.ops import gemm as G
    from miles_b200.ops.norm import add_rms_norm
    from miles_b200.parallel.symm import SymmComm

    H = 2048
    comm = SymmComm(dist.group.WORLD, hidden=H, cap_rows=1024)
    torch.manual_seed(300 + rank)

    def ordered_sum(x):
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        acc = torch.zeros_like(x, dtype=torch.float32)
        for p_ in parts:
            acc += p_.float()
        return acc.to(x.dtype)

    ok = {}
    for M in (1, 64, 512):
        a = torch.randn(M, 1024, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(H, 1024, device="cuda", dtype=torch.bfloat16) * 0.03
        r = torch.randn(M, H, device="cuda", dtype=torch.bfloat16)
        dist.broadcast(r, 0)
        nw = torch.rand(H, device="cuda", dtype=torch.bfloat16) + 0.5
        dist.broadcast(nw, 0)
        part = G.linear(a, w)
        ref = ordered_sum(part)
        ok[f"ar{M}"] = bool(torch.equal(comm.all_reduce(part), ref))
        ok[f"gemm_ar{M}"] = bool(torch.equal(comm.gemm_all_reduce(a, w), ref))
        y_ref, h_ref = add_rms_norm(ref, r, nw, 1e-6)
        y, h = comm.gemm_all_reduce(a, w, res=r, norm_w=nw, eps=1e-6)
        ok[f"gemm_ar_norm{M}"] = bool(torch.equal(y, y_ref) and torch.equal(h, h_ref))
    rows = 128 * world
    x = torch.randn(rows, H, device="cuda", dtype=torch.bfloat16)
    ref = ordered_sum(x)
    ok["rs"] = bool(torch.equal(comm.reduce_scatter(x), ref[rank * 128:(rank + 1) * 128]))
    parts = [torch.empty(100, H, device="cuda", dtype=torch.bfloat16) for _ in range(world)]
    dist.all_gather(parts, x[:100].contiguous())
    ok["ag"] = bool(torch.equal(comm.all_gather(x[:100]), torch.cat(parts)))
    a = torch.randn(rows, 1024, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, 1024, device="cuda", dtype=torch.bfloat16) * 0.03
    ref = ordered_sum(G.linear(a, w))
    ok["gemm_rs"] = bool(torch.equal(comm.gemm_reduce_scatter(a, w), ref[rank * 128:(rank + 1) * 128]))
    check_device_error()
    flags = torch.tensor([int(all(ok.values()))], device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    comm.close()
    if rank == 0:
        torch.save({"ok": bool(flags.item()), "detail": ok}, out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [4, 8])
def test_symm_collectives_n_ranks(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = str(tmp_path / "c.pt")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_n_rank_collectives, args=(free_port(), out, world), nprocs=world, join=True)
    r = torch.load(out)
    print(r)
    assert r["ok"], r["detail"]
