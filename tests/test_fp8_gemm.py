"""Block-scaled fp8 GEMM (tcgen05 kind::f8f6f4) against an fp32 PyTorch GEMM of the dequantised
operands: dense shapes (decode to training sizes), tile-width / batch invariance, grouped MoE
shapes with empty experts, and the fused SwiGLU epilogue."""
import pytest
import torch

from miles_b200.ops import check_device_error
from miles_b200.ops import fp8 as F

pytestmark = pytest.mark.gpu


def _close(out, ref, tol=1e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"rel err {err / scale}"


def test_act_quant_matches_reference():
    torch.manual_seed(0)
    x = (torch.randn(300, 1024, device="cuda") * torch.rand(300, 1, device="cuda") * 5).bfloat16()
    x[3, :128] = 0  # all-zero group: floor scale
    q, s = F.quant_act(x)
    qr, sr = F.quant_act_ref(x)
    # the scale may differ from torch's division by an ulp; the codes then only at ties
    torch.testing.assert_close(s, sr, rtol=2e-7, atol=0)
    same = (q == qr.view(torch.uint8)).float().mean().item()
    assert same > 0.995, same
    check_device_error()


@pytest.mark.parametrize("M,N,K", [(1, 2048, 2048), (7, 4096, 2048), (64, 512, 2048),
                                   (300, 768, 384), (1024, 2048, 768), (4096, 4096, 2048)])
def test_dense(M, N, K):
    torch.manual_seed(1)
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = F.Fp8Weight.from_bf16((torch.randn(N, K, device="cuda") * 0.05).bfloat16())
    xq, xs = F.quant_act(x)
    out = F.fp8_gemm(xq, xs, w, torch.empty(M, N, device="cuda", dtype=torch.bfloat16), M, N)
    torch.cuda.synchronize()
    _close(out, F.fp8_gemm_ref(xq, xs, w, M, N))
    check_device_error()


@pytest.mark.parametrize("bn", [32, 64, 128])
def test_tile_width_and_batch_invariance(bn):
    torch.manual_seed(2)
    M, N, K = 256, 1024, 1024
    x = torch.randn(M, K, device="cuda").bfloat16()
    w = F.Fp8Weight.from_bf16((torch.randn(N, K, device="cuda") * 0.05).bfloat16())
    xq, xs = F.quant_act(x)
    ref = F.fp8_gemm(xq, xs, w, torch.empty(M, N, device="cuda", dtype=torch.bfloat16), M, N, bn=128)
    out = F.fp8_gemm(xq, xs, w, torch.empty(M, N, device="cuda", dtype=torch.bfloat16), M, N, bn=bn)
    assert torch.equal(ref, out)
    for m in (1, 3, 40, 100):
        pq, ps = F.quant_act(x[:m].contiguous())
        part = F.fp8_gemm(pq, ps, w, torch.empty(m, N, device="cuda", dtype=torch.bfloat16), m, N, bn=bn)
        assert torch.equal(part, ref[:m]), m
    check_device_error()


def _grouped_case(E, counts, K, N, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    pad = [((c + 127) // 128) * 128 for c in counts]
    offs = [0]
    for p_ in pad:
        offs.append(offs[-1] + p_)
    Mp = max(offs[-1], 128)
    x = torch.zeros(Mp, K, device="cuda", dtype=torch.bfloat16)
    for e in range(E):
        x[offs[e]:offs[e] + counts[e]] = torch.randn(counts[e], K, device="cuda", generator=g).bfloat16()
    w = F.Fp8Weight.from_bf16((torch.randn(E * N, K, device="cuda", generator=g) * 0.05).bfloat16())
    go = torch.tensor(offs, dtype=torch.int32, device="cuda")
    gc = torch.tensor(counts, dtype=torch.int32, device="cuda")
    return x, w, go, gc, offs, Mp


def test_grouped_with_empty_experts():
    E, K, N = 8, 2048, 768
    counts = [5, 0, 300, 128, 0, 1, 257, 40]
    x, w, go, gc, offs, Mp = _grouped_case(E, counts, K, N, 3)
    xq, xs = F.quant_act(x)
    out = torch.zeros(Mp, N, device="cuda", dtype=torch.bfloat16)
    F.fp8_gemm(xq, xs, w, out, Mp, N, mode=1, group_offsets=go, group_counts=gc, num_groups=E,
               b_rows_per_group=N)
    torch.cuda.synchronize()
    a = xq.view(torch.float8_e4m3fn).float().view(Mp, K // 128, 128) * xs.t()[..., None]
    a = a.view(Mp, K)
    wd = w.dequant().view(E, N, K)
    for e in range(E):
        r0, c = offs[e], counts[e]
        if c == 0:
            continue
        _close(out[r0:r0 + c], a[r0:r0 + c] @ wd[e].t())
    check_device_error()


def test_grouped_swiglu():
    E, K, Fdim = 4, 2048, 768
    counts = [130, 0, 7, 64]
    x, w, go, gc, offs, Mp = _grouped_case(E, counts, K, 2 * Fdim, 4)
    xq, xs = F.quant_act(x)
    out = torch.zeros(Mp, Fdim, device="cuda", dtype=torch.bfloat16)
    gu = torch.zeros(Mp, 2 * Fdim, device="cuda", dtype=torch.bfloat16)
    F.fp8_gemm(xq, xs, w, out, Mp, 2 * Fdim, mode=1, group_offsets=go, group_counts=gc,
               num_groups=E, b_rows_per_group=2 * Fdim, swiglu_f=Fdim, gu=gu)
    # the plain grouped product gives [gate | up]; SwiGLU of its bf16 values must match bitwise
    plain = torch.zeros(Mp, 2 * Fdim, device="cuda", dtype=torch.bfloat16)
    F.fp8_gemm(xq, xs, w, plain, Mp, 2 * Fdim, mode=1, group_offsets=go, group_counts=gc,
               num_groups=E, b_rows_per_group=2 * Fdim)
    torch.cuda.synchronize()
    for e in range(E):
        r0, c = offs[e], counts[e]
        if c == 0:
            continue
        assert torch.equal(gu[r0:r0 + c], plain[r0:r0 + c])
        g_, u_ = plain[r0:r0 + c, :Fdim].float(), plain[r0:r0 + c, Fdim:].float()
        ref = (g_ / (1 + torch.exp(-g_))).bfloat16().float() * u_
        _close(out[r0:r0 + c], ref, tol=1e-2)
    check_device_error()


def test_linear_wrapper():
    torch.manual_seed(5)
    x = torch.randn(33, 2048, device="cuda").bfloat16()
    wb = (torch.randn(4096, 2048, device="cuda") * 0.05).bfloat16()
    w = F.Fp8Weight.from_bf16(wb)
    y = F.fp8_linear(x, w)
    # fp8 error against the bf16 product stays at the e4m3 level
    ref = x.float() @ wb.float().t()
    _close(y, ref, tol=6e-2)
    check_device_error()


def test_fp8_model_rollout_train_parity():
    """Unified fp8: with the block-scaled fp8 copies enabled, the rollout engine's decode
    log-probs (and routing) equal the training forward's bit for bit, and a weight update
    re-quantises the copies in place."""
    import numpy as np

    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.ops.logprob import lm_head_logprob

    cfg = preset("small-moe")
    m = Transformer(cfg, device="cuda", seed=0)
    m.enable_fp8()
    try:
        assert "layers.0.mlp.experts.w1" in m.fp8 and "layers.0.self_attn.qkv_proj.weight" in m.fp8
        rng = np.random.default_rng(0)
        reqs = [GenRequest(rng.integers(0, cfg.vocab_size, int(rng.integers(5, 90))).tolist(),
                           int(rng.integers(3, 30)), seed=11 + i, rid=i, return_routed_experts=True)
                for i in range(10)]
        eng = RolloutEngine(m, max_batch=8, num_pages=128, max_pages_per_seq=4, steps_per_sync=8)
        outs = eng.generate(reqs)
        for r, o in zip(reqs, outs):
            toks = r.prompt + o.tokens
            rec = []
            with torch.no_grad():
                h = m.forward_train(torch.tensor(toks, dtype=torch.int32, device="cuda"),
                                    VarlenMeta([0, len(toks)], "cuda"), record_experts=rec)
                sel = torch.arange(len(r.prompt) - 1, len(toks) - 1, device="cuda")
                lp, _ = lm_head_logprob(h.index_select(0, sel), m.lm_head_weight(),
                                        torch.tensor(o.tokens, dtype=torch.int32, device="cuda"), 1.0, 4096)
            assert torch.equal(lp.float().cpu(), torch.tensor(o.logprobs, dtype=torch.float32))
            ex = torch.stack(rec, 1)[: len(toks) - 1].cpu().numpy()
            assert (o.routed_experts == ex).all()
        # training forward + backward through the fp8 forward: finite gradients on bf16 weights
        toks = torch.tensor(reqs[0].prompt + outs[0].tokens, dtype=torch.int32, device="cuda")
        h = m.forward_train(toks, VarlenMeta([0, toks.numel()], "cuda"))
        h.float().square().mean().backward()
        g = m.params["layers.0.mlp.experts.w1"].grad
        g2 = getattr(m.params["layers.0.mlp.experts.w1"], "main_grad", None)
        assert (g is not None and torch.isfinite(g).all()) or g2 is not None
        # a weight update bumps the version; the next forward re-quantises in place
        w8 = m.fp8["layers.0.self_attn.o_proj.weight"]
        ptr, before = w8.q.data_ptr(), w8.q.clone()
        with torch.no_grad():
            m.params["layers.0.self_attn.o_proj.weight"].mul_(2.0)
        m.weight_version += 1
        m.sync_fp8()
        assert w8.q.data_ptr() == ptr and torch.equal(w8.q, before)  # x2 only moves the scales
        check_device_error()
    finally:
        m.disable_fp8()
