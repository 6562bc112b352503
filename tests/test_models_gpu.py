"""MLA, DSA and Gated DeltaNet model families on a B200 (bf16, the native GEMM / norm kernels
plus the PyTorch attention variants): engine decode (CUDA graphs) reproduces the training
forward's greedy tokens and log-probs within bf16 tolerance, and a backward runs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["tiny-mla", "tiny-dsa", "tiny-gdn"])
def test_family_decode_matches_forward(name):
    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops import check_device_error
    from miles_b200.ops.attention import VarlenMeta
    from miles_b200.ops.logprob import lm_head_logprob

    cfg = preset(name)
    m = Transformer(cfg, device="cuda", seed=0)
    eng = RolloutEngine(m, max_batch=4, num_pages=64, max_pages_per_seq=8, use_cuda_graph=True)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab_size, n).tolist() for n in (12, 70, 33)]
    outs = eng.generate([GenRequest(p, 8, temperature=1.0, seed=3 + i, rid=i) for i, p in enumerate(prompts)])
    diffs = []
    with torch.no_grad():
        for p, o in zip(prompts, outs):
            toks = p + o.tokens
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32, device="cuda"),
                                VarlenMeta([0, len(toks)], "cuda"))
            sel = torch.arange(len(p) - 1, len(toks) - 1, device="cuda")
            lp, _ = lm_head_logprob(h.index_select(0, sel), m.lm_head_weight(),
                                    torch.tensor(o.tokens, dtype=torch.int32, device="cuda"), 1.0, 4096)
            diffs.append((lp.float().cpu() - torch.tensor(o.logprobs)).abs())
    d = torch.cat(diffs)
    # bf16 activations; the attention variants run different op orders in decode and training
    assert d.mean() < 0.05 and d.max() < 0.5, (float(d.mean()), float(d.max()))
    m.recompute = False
    toks = torch.randint(0, cfg.vocab_size, (96,), device="cuda", dtype=torch.int32)
    h = m.forward_train(toks, VarlenMeta([0, 40, 96], "cuda"))
    h.float().pow(2).mean().backward()
    assert all(p.grad is None or torch.isfinite(p.grad.float()).all() for p in m.params.values())
    check_device_error()


def test_gdn_decode_kernel_matches_reference():
    """csrc/gdn.cu: in-place state update and outputs equal the PyTorch step (fp32), with state
    rows addressed through the row table and two steps in a row."""
    from miles_b200.models.gdn import gdn_step_ref
    from miles_b200.ops._lib import lib

    torch.manual_seed(0)
    B, nv, dk, dv, R = 5, 4, 128, 128, 8
    rows = torch.tensor([3, 0, 7, 5, 1], dtype=torch.int64, device="cuda")
    S = torch.randn(R, nv, dk, dv, device="cuda") * 0.1
    S_ref = S.clone()
    for _ in range(2):
        q = torch.nn.functional.normalize(torch.randn(B, nv, dk, device="cuda"), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(B, nv, dk, device="cuda"), dim=-1)
        v = torch.randn(B, nv, dv, device="cuda")
        beta = torch.rand(B, nv, device="cuda")
        g = -torch.rand(B, nv, device="cuda")
        o = torch.empty(B, nv, dv, device="cuda")
        lib().gdn_decode(q, k, v, beta, g, rows, S, o, dk ** -0.5)
        o_ref, s_new = gdn_step_ref(q, k, v, beta, g, S_ref[rows], dk)
        S_ref[rows] = s_new
        torch.cuda.synchronize()
        assert torch.allclose(o, o_ref, atol=1e-4, rtol=1e-4)
        assert torch.allclose(S, S_ref, atol=1e-5, rtol=1e-4)


@pytest.mark.parametrize("with_bias", [False, True])
def test_mla_decode_kernel_matches_reference(with_bias):
    """csrc/mla_decode.cu against the PyTorch absorbed decode over gathered cache rows."""
    from miles_b200.ops._lib import lib

    torch.manual_seed(0)
    B, nh, r, dr, extra, P = 3, 4, 512, 64, 32, 5
    width = r + dr + extra
    slots = 16 * 64
    cache = (torch.randn(slots, 1, width, device="cuda") * 0.5).to(torch.bfloat16)
    pt = torch.stack([torch.randperm(16, device="cuda")[:P] for _ in range(B)]).int()
    ctx = torch.tensor([1, 200, P * 64], dtype=torch.int32, device="cuda")
    q_lat = torch.randn(B, nh, r, device="cuda")
    q_pe = torch.randn(B, nh, dr, device="cuda")
    maxk = P * 64
    bias = None
    if with_bias:
        bias = torch.zeros(B, maxk, device="cuda")
        bias[:, 1::3] = float("-inf")
    out = torch.empty(B, nh, r, device="cuda")
    scale = 0.07
    lib().mla_decode(q_lat, q_pe, cache[:, 0, :], pt, ctx, bias, scale, out)
    t = torch.arange(maxk, device="cuda")
    rows = pt.long()[:, t // 64] * 64 + (t % 64)[None, :]
    lat = cache[:, 0, :].index_select(0, rows.reshape(-1)).view(B, maxk, width).float()
    sc = (torch.einsum("bhc,btc->bht", q_lat, lat[..., :r]) +
          torch.einsum("bhd,btd->bht", q_pe, lat[..., r:r + dr])) * scale
    if bias is not None:
        sc = sc + bias[:, None, :]
    sc = sc.masked_fill((t[None, :] >= ctx[:, None].long())[:, None, :], float("-inf"))
    ref = torch.einsum("bht,btc->bhc", torch.softmax(sc, -1), lat[..., :r])
    torch.cuda.synchronize()
    assert torch.allclose(out, ref, atol=2e-4, rtol=1e-3), (out - ref).abs().max()
