"""Single-kernel workloads for profiling (ncu) and timing:

    python -m miles_b200.profiling.cases <case>

cases: gemm_dense (8192x6144x2048 bf16 tcgen05 GEMM), gemm_grouped_decode (gate_up + SwiGLU of a
64-token MoE decode step, 128 experts), attn_fwd (2 x 4096 tokens, 32 q / 4 kv heads), attn_bwd
(same, backward), attn_decode (64 sequences x 4096 keys, paged).
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
elif case == "attn_decode":
    from miles_b200.ops.attention import decode_attention
    B, nq, nkv, ctx, P = 64, 32, 4, 4096, 64
    pages = B * ctx // P
    kc = torch.randn(pages * P, nkv, 128, device='cuda', dtype=torch.bfloat16)
    vc = torch.randn(pages * P, nkv, 128, device='cuda', dtype=torch.bfloat16)
    pt = torch.randperm(pages, device='cuda').int().view(B, ctx // P).contiguous()
    q = torch.randn(B, nq, 128, device='cuda', dtype=torch.bfloat16)
    lens = torch.full((B,), ctx, dtype=torch.int32, device='cuda')
    for _ in range(4): decode_attention(q, kc, vc, pt, lens)
torch.cuda.synchronize()
print("ok", case)
