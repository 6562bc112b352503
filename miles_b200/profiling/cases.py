"""Single-kernel workloads for profiling (ncu) and timing:

    python -m miles_b200.profiling.cases <case>

cases: gemm_dense (8192x6144x2048 bf16 tcgen05 GEMM), gemm_grouped_decode (gate_up + SwiGLU of a
64-token MoE decode step, 128 experts), attn_fwd (2 x 4096 tokens, 32 q / 4 kv heads), attn_bwd
(same, backward), attn_decode (64 sequences x 4096 keys, paged), symm_ar_norm (one-rank group:
GEMM storing into the symmetric staging + reduce/residual/RMSNorm kernel, 4096 x 2048 output),
ep_dispatch_combine (one-rank expert-parallel layer through the peer-memory dispatch / combine
kernels: 4096 tokens, top-8 of 128 experts, forward and backward), rl_step (Qwen3-30B-A3B widths
with 2 layers: one training step of 8192 packed tokens -- norms, RoPE, router, MoE permute /
combine, SwiGLU, log-prob, policy loss, Adam -- and 8 engine decode steps of 64 sequences --
decode-state prep / commit, fused route + dispatch, sampler; the small-kernel profiles use it),
rl_math (GRPO advantages and chunked GAE over 64k tokens), fp8_gemm_dense (block-scaled fp8
GEMM 8192x6144x2048 with its 1 x 128 activation quantisation), fp8_grouped_decode (the
gemm_grouped_decode step on fp8 expert weights), attn_decode256 (256 sequences x 4096 keys),
small_kernels (the memory-bound kernels of a training / decode step on inputs larger than L2, a
few GB in total: RMSNorm fwd / bwd, QK-norm + RoPE fwd / bwd, SwiGLU fwd / bwd, router fwd / bwd,
MoE permute plan / gather / combine, LM-head log-prob / entropy, sampler, policy loss, Adam,
fp8 activation and block quantisation), family_decode (engine decode of 64 sequences on a
2-layer DeepSeek-V3-width MLA model and the tiny Gated DeltaNet hybrid: the absorbed-MLA and
GDN decode kernels; plus the fp8 block dequantisation and the RL advantage kernels).
"""
import sys

import torch
case = sys.argv[1]
torch.manual_seed(0)
if case == "gemm_dense":
    from miles_b200.ops import gemm as G
    a = torch.randn(8192, 2048, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(6144, 2048, device="cuda", dtype=torch.bfloat16)
    for _ in range(4): G.matmul_nt(a, b)
elif case == "fp8_gemm_dense":
    from miles_b200.ops import fp8 as F8
    a = torch.randn(8192, 2048, device="cuda", dtype=torch.bfloat16)
    w = F8.Fp8Weight.from_bf16(torch.randn(6144, 2048, device="cuda", dtype=torch.bfloat16))
    out = torch.empty(8192, 6144, device="cuda", dtype=torch.bfloat16)
    for _ in range(4):
        aq, sa = F8.quant_act(a)
        F8.fp8_gemm(aq, sa, w, out, 8192, 6144)
elif case == "fp8_grouped_decode":
    from miles_b200.ops import fp8 as F8
    from miles_b200.ops.moe import MoEPlan
    E, K, F, k, T = 128, 2048, 768, 8, 64
    idx = torch.stack([torch.randperm(E, device='cuda')[:k] for _ in range(T)]).int()
    plan = MoEPlan(idx, E)
    x = torch.randn(T, K, device='cuda', dtype=torch.bfloat16)
    xs = plan.gather(x)
    w1 = F8.Fp8Weight.from_bf16(torch.randn(E * 2 * F, K, device='cuda', dtype=torch.bfloat16))
    w2 = F8.Fp8Weight.from_bf16(torch.randn(E * K, F, device='cuda', dtype=torch.bfloat16))
    for _ in range(4):
        F8.fp8_experts(xs, w1, w2, plan.offsets, plan.counts, E, F, K, save_gu=False)
elif case == "small_kernels":
    from miles_b200.ops import fp8 as F8
    from miles_b200.ops.logprob import lm_head_logprob, sample_from_hidden
    from miles_b200.ops.moe import RouterCfg, moe_experts
    from miles_b200.ops.norm import qk_norm_rope, rms_norm, rope_tables, swiglu
    from miles_b200.ops.optim import adam_
    from miles_b200.ops.quant import fp8_block_quant
    from miles_b200.ops.rl import PolicyLossCfg, policy_loss
    T, H, E, F = 32768, 2048, 128, 768

    def mark(name):
        torch.cuda.synchronize()
        print("ok", name, flush=True)
    for _ in range(2):
        x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        w = torch.ones(H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        rms_norm(x, w).sum().backward()
        mark("rmsnorm")
        qkv = torch.randn(T, 5120, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        cos, sin = rope_tables(8192, 128, 1e6, "cuda")
        pos = (torch.arange(T, device="cuda") % 8192).int()
        qw = torch.ones(128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        q, k, v = qk_norm_rope(qkv, qw, qw, pos, cos, sin, 32, 4)
        (q.float().sum() + k.float().sum() + v.float().sum()).backward()
        mark("qk_norm_rope")
        gu = torch.randn(T, 2 * F, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        swiglu(gu).sum().backward()
        mark("swiglu")
        xm = torch.randn(8192, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        rw = torch.randn(E, H, device="cuda", dtype=torch.bfloat16, requires_grad=True) * 0.02
        w1 = torch.randn(E, 2 * F, H, device="cuda", dtype=torch.bfloat16) * 0.02
        w2 = torch.randn(E, H, F, device="cuda", dtype=torch.bfloat16) * 0.02
        moe_experts(xm, rw, w1, w2, RouterCfg(E, 8)).float().sum().backward()
        mark("moe")
        hh = torch.randn(2048, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        Wv = torch.randn(151936, H, device="cuda", dtype=torch.bfloat16) * 0.02
        tg = torch.randint(0, 151936, (2048,), device="cuda", dtype=torch.int32)
        lp, ent = lm_head_logprob(hh, Wv, tg)
        n = lp.numel()
        loss, _ = policy_loss(lp, lp.detach(), torch.randn(n, device="cuda"),
                              torch.full((n,), 1.0 / n, device="cuda"), PolicyLossCfg(use_tis=True),
                              rollout_logp=lp.detach() - 0.01)
        loss.backward()
        mark("logprob+policy_loss")
        hs = torch.randn(256, H, device="cuda", dtype=torch.bfloat16)
        sample_from_hidden(hs, Wv, torch.ones(256, device="cuda"),
                           torch.arange(256, device="cuda", dtype=torch.int64),
                           torch.zeros(256, device="cuda", dtype=torch.int32))
        mark("sample")
        N = 1 << 26
        prm = torch.randn(N, device="cuda").bfloat16()
        adam_(prm, torch.randn(N, device="cuda").bfloat16(), torch.zeros(N, device="cuda"),
              torch.zeros(N, device="cuda"), master=torch.zeros(N, device="cuda"), lr=1e-6)
        mark("adam")
        F8.quant_act(torch.randn(T, H, device="cuda", dtype=torch.bfloat16))
        mark("act_quant")
        fp8_block_quant(torch.randn(6144, H, device="cuda", dtype=torch.bfloat16))
        del x, qkv, gu, xm, Wv
        torch.cuda.synchronize()
elif case == "family_decode":
    import dataclasses

    import numpy as np

    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.quant import fp8_block_dequant, fp8_block_quant
    from miles_b200.ops.rl import gae, grpo_advantages
    dev = sys.argv[2] if len(sys.argv) > 2 else "cuda"
    dt = torch.bfloat16 if dev == "cuda" else torch.float32
    rng = np.random.default_rng(0)
    for name, layers, ctx in (("dsv3-small", 2, 1024), ("tiny-gdn", None, 512)):
        cfg = preset(name)
        if layers:
            cfg = dataclasses.replace(cfg, num_layers=layers)
        m = Transformer(cfg, device=dev, dtype=dt, seed=0)
        eng = RolloutEngine(m, max_batch=64, num_pages=64 * (ctx // 64 + 2), max_pages_per_seq=ctx // 64 + 2,
                            use_cuda_graph=False)
        eng.generate([GenRequest(rng.integers(0, cfg.vocab_size, ctx).tolist(), 8, seed=i, rid=i)
                      for i in range(64)])
        del eng, m
    q, sc = fp8_block_quant(torch.randn(6144, 2048, device=dev).to(dt))
    fp8_block_dequant(q, sc)
    n = 1 << 16
    grpo_advantages(torch.rand(4096, device=dev), 8)
    gae(torch.randn(n, device=dev), torch.randn(n, device=dev), list(range(0, n + 1, 1024)), 1.0, 0.95)
elif case == "gemm_grouped_decode":
    from miles_b200.ops import gemm as G
    from miles_b200.ops.moe import MoEPlan
    E, K, F, k, T = 128, 2048, 768, 8, 64
    idx = torch.stack([torch.randperm(E, device='cuda')[:k] for _ in range(T)]).int()
    plan = MoEPlan(idx, E)
    x = torch.randn(T, K, device='cuda', dtype=torch.bfloat16)
    xs = plan.gather(x)
    w1 = torch.randn(E, 2 * F, K, device='cuda', dtype=torch.bfloat16)
    for _ in range(4): G.grouped_nt_swiglu(xs, w1, plan.offsets, n_rows=T * k, counts=plan.counts)
elif case in ("attn_fwd", "attn_bwd"):
    from miles_b200.ops.attention import VarlenMeta, varlen_attention
    nq, nkv, D = 32, 4, 128
    lens = [4096] * 2
    cu = [0]
    for L in lens: cu.append(cu[-1] + L)
    T = cu[-1]
    q = torch.randn(T, nq, D, device='cuda', dtype=torch.bfloat16, requires_grad=case == "attn_bwd")
    k_ = torch.randn(T, nkv, D, device='cuda', dtype=torch.bfloat16, requires_grad=case == "attn_bwd")
    v = torch.randn(T, nkv, D, device='cuda', dtype=torch.bfloat16, requires_grad=case == "attn_bwd")
    meta = VarlenMeta(cu, 'cuda')
    for _ in range(2):
        o = varlen_attention(q, k_, v, meta)
        if case == "attn_bwd":
            o.backward(torch.ones_like(o))
elif case in ("attn_decode", "attn_decode256"):
    from miles_b200.ops.attention import decode_attention
    B, nq, nkv, ctx, P = 64 if case == "attn_decode" else 256, 32, 4, 4096, 64
    pages = B * ctx // P
    kc = torch.randn(pages * P, nkv, 128, device='cuda', dtype=torch.bfloat16)
    vc = torch.randn(pages * P, nkv, 128, device='cuda', dtype=torch.bfloat16)
    pt = torch.randperm(pages, device='cuda').int().view(B, ctx // P).contiguous()
    q = torch.randn(B, nq, 128, device='cuda', dtype=torch.bfloat16)
    lens = torch.full((B,), ctx, dtype=torch.int32, device='cuda')
    for _ in range(4): decode_attention(q, kc, vc, pt, lens)
elif case == "rl_step":
    import dataclasses

    import numpy as np

    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.rl import PolicyLossCfg
    from miles_b200.trainer.actor import Actor, ActorConfig, TrainItem
    cfg = dataclasses.replace(preset("qwen3-30b-a3b"), num_layers=2)
    m = Transformer(cfg, device="cuda", seed=0)
    rng = np.random.default_rng(0)
    items = [TrainItem(rng.integers(0, cfg.vocab_size, 1024).tolist(), 256, advantage=1.0,
                       rollout_logp=(-rng.random(768)).tolist()) for _ in range(8)]
    a = Actor(m, ActorConfig(max_tokens_per_gpu=8192, optimizer_placement="device",
                             loss=PolicyLossCfg(use_tis=True, tis_clip=2.0)))
    for _ in range(2):
        a.train_step(items)
    eng = RolloutEngine(m, max_batch=64, num_pages=64 * 24, max_pages_per_seq=24, use_cuda_graph=False)
    eng.generate([GenRequest(rng.integers(0, cfg.vocab_size, 1024).tolist(), 8, seed=i, rid=i,
                             return_routed_experts=True) for i in range(64)])
elif case == "rl_math":
    from miles_b200.ops.rl import gae, grpo_advantages
    r = torch.rand(4096, device="cuda")
    n = 1 << 16
    rew, val = torch.randn(n, device="cuda"), torch.randn(n, device="cuda")
    cu = list(range(0, n + 1, 1024))
    for _ in range(3):
        grpo_advantages(r, 8)
        gae(rew, val, cu, 1.0, 0.95)
elif case in ("symm_ar_norm", "ep_dispatch_combine"):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:29731", rank=0, world_size=1)
    if case == "symm_ar_norm":
        from miles_b200.parallel.symm import SymmComm
        H, K, M = 2048, 4096, 4096
        comm = SymmComm(dist.group.WORLD, hidden=H, cap_rows=M)
        a = torch.randn(M, K, device='cuda', dtype=torch.bfloat16)
        w = torch.randn(H, K, device='cuda', dtype=torch.bfloat16) * 0.02
        r = torch.randn(M, H, device='cuda', dtype=torch.bfloat16)
        nw = torch.ones(H, device='cuda', dtype=torch.bfloat16)
        for _ in range(3): comm.gemm_all_reduce(a, w, res=r, norm_w=nw, eps=1e-6)
    else:
        from miles_b200.ops.moe import RouterCfg
        from miles_b200.parallel.ep import EPContext, moe_experts_ep
        E, k, H, I, T = 128, 8, 2048, 768, 4096
        ep = EPContext(dist.group.WORLD, E, "peer", H, k, cap_tokens=T)
        x = torch.randn(T, H, device='cuda', dtype=torch.bfloat16, requires_grad=True)
        rw = (torch.randn(E, H, device='cuda', dtype=torch.bfloat16) * 0.02).requires_grad_()
        w1 = (torch.randn(E, 2 * I, H, device='cuda', dtype=torch.bfloat16) * 0.02).requires_grad_()
        w2 = (torch.randn(E, H, I, device='cuda', dtype=torch.bfloat16) * 0.02).requires_grad_()
        cfg = RouterCfg(E, k)
        for _ in range(2):
            y = moe_experts_ep(x, rw, w1, w2, cfg, ep)
            y.backward(torch.ones_like(y))
    dist.destroy_process_group()
torch.cuda.synchronize()
print("ok", case)
