"""Numerics of the sm_100a kernels against plain PyTorch fp32 references of the same ops."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF = torch.bfloat16


def rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / (b.abs().max() + 1e-6)).item()


def test_rmsnorm_fwd_bwd():
    from miles_b200.ops.norm import add_rms_norm, rms_norm, rms_norm_ref
    torch.manual_seed(0)
    for H in (2048, 2560, 4096):
        x = torch.randn(37, H, device=DEV, dtype=BF, requires_grad=True)
        w = (1 + 0.1 * torch.randn(H, device=DEV)).to(BF).requires_grad_()
        y = rms_norm(x, w, 1e-6)
        yr = rms_norm_ref(x.detach().float(), w.detach().float(), 1e-6)
        assert rel(y, yr) < 1e-2
        g = torch.randn_like(y)
        y.backward(g)
        xr = x.detach().float().requires_grad_()
        wr = w.detach().float().requires_grad_()
        ((xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6)) * wr).backward(g.float())
        assert rel(x.grad, xr.grad) < 2e-2
        assert rel(w.grad, wr.grad) < 2e-2
    res = torch.randn(5, 2048, device=DEV, dtype=BF)
    x = torch.randn(5, 2048, device=DEV, dtype=BF)
    w = torch.ones(2048, device=DEV, dtype=BF)
    y, h = add_rms_norm(x, res, w)
    assert torch.equal(h, (x.float() + res.float()).to(BF))
    assert rel(y, rms_norm_ref(h, w, 1e-6)) < 1e-2


def test_qk_norm_rope():
    from miles_b200.ops.norm import qk_norm_rope, qk_norm_rope_ref, rope_tables
    torch.manual_seed(1)
    T, nq, nkv = 50, 8, 2
    cos, sin = rope_tables(4096, 128, 1e6, DEV)
    qkv = torch.randn(T, (nq + 2 * nkv) * 128, device=DEV, dtype=BF, requires_grad=True)
    qw = (1 + 0.1 * torch.randn(128, device=DEV)).to(BF).requires_grad_()
    kw = (1 + 0.1 * torch.randn(128, device=DEV)).to(BF).requires_grad_()
    pos = torch.randint(0, 4000, (T,), device=DEV, dtype=torch.int32)
    q, k, v = qk_norm_rope(qkv, qw, kw, pos, cos, sin, nq, nkv)
    qr, kr, vr = qk_norm_rope_ref(qkv.detach(), qw.detach(), kw.detach(), pos, cos, sin, nq, nkv, 1e-6)
    assert rel(q, qr) < 1e-2 and rel(k, kr) < 1e-2 and torch.equal(v, vr)
    gq, gk, gv = torch.randn_like(q), torch.randn_like(k), torch.randn_like(v)
    torch.autograd.backward([q, k, v], [gq, gk, gv])
    x = qkv.detach().float().requires_grad_()
    qwf, kwf = qw.detach().float().requires_grad_(), kw.detach().float().requires_grad_()
    xx = x.view(T, nq + 2 * nkv, 128)

    def nr(t, ww):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * ww

    def rope(t):
        c = cos[pos.long()][:, None]
        s = sin[pos.long()][:, None]
        a, b = t[..., :64], t[..., 64:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    q2, k2, v2 = rope(nr(xx[:, :nq], qwf)), rope(nr(xx[:, nq:nq + nkv], kwf)), xx[:, nq + nkv:]
    torch.autograd.backward([q2, k2, v2], [gq.float(), gk.float(), gv.float()])
    assert rel(qkv.grad, x.grad) < 3e-2
    assert rel(qw.grad, qwf.grad) < 3e-2 and rel(kw.grad, kwf.grad) < 3e-2


def test_swiglu():
    from miles_b200.ops.norm import swiglu
    torch.manual_seed(2)
    gu = torch.randn(33, 2 * 768, device=DEV, dtype=BF, requires_grad=True)
    y = swiglu(gu)
    g = gu.detach().float().requires_grad_()
    yr = torch.nn.functional.silu(g[:, :768]) * g[:, 768:]
    assert rel(y, yr) < 1e-2
    d = torch.randn_like(y)
    y.backward(d)
    yr.backward(d.float())
    assert rel(gu.grad, g.grad) < 2e-2


@pytest.mark.parametrize("score_fn", ["softmax", "sigmoid"])
def test_router(score_fn):
    from miles_b200.ops._lib import lib
    from miles_b200.ops.moe import RouterCfg, route_ref
    torch.manual_seed(3)
    T, E, k = 100, 64, 6
    sig = score_fn == "sigmoid"
    cfg = RouterCfg(E, k, score_fn, True, n_group=8 if sig else 1, topk_group=4 if sig else 1,
                    scale=2.5 if sig else 1.0)
    logits = torch.randn(T, E, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1 if sig else None
    idx = torch.empty(T, k, dtype=torch.int32, device=DEV)
    w = torch.empty(T, k, device=DEV)
    lib().router_fwd(logits, bias, None, idx, w, k, cfg.score_fn, True, cfg.n_group, cfg.topk_group, cfg.scale)
    ir, wr = route_ref(logits, cfg, bias)
    assert torch.equal(idx, ir)
    assert rel(w, wr) < 1e-5
    idx2 = torch.empty_like(idx)
    w2 = torch.empty_like(w)
    lib().router_fwd(logits, bias, idx, idx2, w2, k, cfg.score_fn, True, cfg.n_group, cfg.topk_group, cfg.scale)
    assert torch.equal(idx2, idx) and torch.equal(w2, w)
    dw = torch.randn(T, k, device=DEV)
    dl = torch.empty(T, E, dtype=BF, device=DEV)
    lib().router_bwd(logits, idx, dw, dl, cfg.score_fn, True, cfg.scale)
    lf = logits.clone().requires_grad_()
    sc = lf.softmax(-1) if not sig else lf.sigmoid()
    sel = sc.gather(1, idx.long())
    ww = sel / sel.sum(-1, keepdim=True) * cfg.scale
    ww.backward(dw)
    assert rel(dl, lf.grad) < 2e-2


def test_moe_layer():
    from miles_b200.ops.moe import RouterCfg, moe_experts, moe_ref
    torch.manual_seed(4)
    T, H, I, E, k = 300, 256, 128, 16, 4
    cfg = RouterCfg(E, k)
    x = (torch.randn(T, H, device=DEV) * 0.5).to(BF).requires_grad_()
    rw = (torch.randn(E, H, device=DEV) * 0.05).to(BF).requires_grad_()
    w1 = (torch.randn(E, 2 * I, H, device=DEV) * 0.05).to(BF).requires_grad_()
    w2 = (torch.randn(E, H, I, device=DEV) * 0.05).to(BF).requires_grad_()
    rec = []
    y = moe_experts(x, rw, w1, w2, cfg, record=rec.append)
    yr, idx_r = moe_ref(x.detach(), rw.detach(), w1.detach(), w2.detach(), cfg)
    assert torch.equal(rec[0], idx_r)
    assert rel(y, yr) < 2e-2
    y2 = moe_experts(x.detach(), rw.detach(), w1.detach(), w2.detach(), cfg)
    assert torch.equal(y.detach(), y2)
    g = torch.randn_like(y)
    y.backward(g)
    xf = x.detach().float().requires_grad_()
    rwf = rw.detach().float().requires_grad_()
    w1f = w1.detach().float().requires_grad_()
    w2f = w2.detach().float().requires_grad_()
    sc = (xf @ rwf.t()).softmax(-1)
    sel = sc.gather(1, idx_r.long())
    wts = sel / sel.sum(-1, keepdim=True)
    out = torch.zeros(T, H, device=DEV)
    for e in range(E):
        tok, slot = (idx_r == e).nonzero(as_tuple=True)
        if tok.numel():
            gu = xf[tok] @ w1f[e].t()
            a = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
            out = out.index_add(0, tok, wts[tok, slot][:, None] * (a @ w2f[e].t()))
    out.backward(g.float())
    assert rel(x.grad, xf.grad) < 5e-2
    assert rel(w1.grad, w1f.grad) < 5e-2
    assert rel(w2.grad, w2f.grad) < 5e-2
    assert rel(rw.grad, rwf.grad) < 5e-2


def _packed(lens, nq, nkv, seed=5):
    torch.manual_seed(seed)
    T = sum(lens)
    q = torch.randn(T, nq, 128, device=DEV, dtype=BF)
    k = torch.randn(T, nkv, 128, device=DEV, dtype=BF)
    v = torch.randn(T, nkv, 128, device=DEV, dtype=BF)
    cu = [0]
    for L in lens:
        cu.append(cu[-1] + L)
    return q, k, v, cu


def test_attention_fwd_bwd():
    from miles_b200.ops.attention import VarlenMeta, attention_ref, varlen_attention
    q, k, v, cu = _packed([1, 63, 64, 65, 200, 7, 1300], 8, 2)
    meta = VarlenMeta(cu, DEV)
    q.requires_grad_(); k.requires_grad_(); v.requires_grad_()
    o = varlen_attention(q, k, v, meta)
    qf, kf, vf = (t.detach().float().requires_grad_() for t in (q, k, v))
    orf = attention_ref(qf, kf, vf, cu)
    assert rel(o, orf) < 2e-2
    g = torch.randn_like(o)
    o.backward(g)
    orf.backward(g.float())
    assert rel(q.grad, qf.grad) < 3e-2
    assert rel(k.grad, kf.grad) < 3e-2
    assert rel(v.grad, vf.grad) < 3e-2


def test_decode_matches_prefill_bitwise():
    """Rollout decode rows are bitwise equal to the corresponding training-forward rows."""
    from miles_b200.ops.attention import VarlenMeta, decode_attention, varlen_attention
    nq, nkv = 8, 2
    lens = [5, 64, 130, 2500, 1025, 1024]
    q, k, v, cu = _packed(lens, nq, nkv, seed=6)
    meta = VarlenMeta(cu, DEV)
    o = varlen_attention(q, k, v, meta)
    B = len(lens)
    max_pages = 40
    nslots = B * max_pages * 64
    # stale cache contents (finite: the engine zero-initialises its cache) must not leak in
    kc = (torch.randn(nslots, nkv, 128, device=DEV) * 100).to(BF)
    vc = (torch.randn(nslots, nkv, 128, device=DEV) * 100).to(BF)
    pt = torch.arange(B * max_pages, dtype=torch.int32, device=DEV).view(B, max_pages).flip(1).contiguous()
    for b, L in enumerate(lens):
        t = torch.arange(L, device=DEV)
        slots = pt[b].long()[t // 64] * 64 + t % 64
        kc[slots] = k[cu[b]:cu[b + 1]]
        vc[slots] = v[cu[b]:cu[b + 1]]
    qd = torch.stack([q[cu[b + 1] - 1] for b in range(B)])
    ctx = torch.tensor(lens, dtype=torch.int32, device=DEV)
    od = decode_attention(qd, kc, vc, pt, ctx)
    for b in range(B):
        assert torch.equal(od[b], o[cu[b + 1] - 1]), b


def test_logprob_and_sampler_parity():
    from miles_b200.ops.logprob import lm_head_logprob, logprob_ref, sample_from_hidden
    torch.manual_seed(7)
    n, H, V = 70, 256, 5000
    h = torch.randn(n, H, device=DEV, dtype=BF, requires_grad=True)
    W = (torch.randn(V, H, device=DEV) * 0.05).to(BF).requires_grad_()
    tgt = torch.randint(0, V, (n,), device=DEV, dtype=torch.int32)
    for temp in (1.0, 0.7):
        lp, ent = lm_head_logprob(h, W, tgt, temp, chunk=32)
        lr, er = logprob_ref(h.detach(), W.detach(), tgt, temp)
        assert (lp - lr).abs().max().item() < 2e-3
        assert (ent - er).abs().max().item() < 2e-3
    lp, ent = lm_head_logprob(h, W, tgt, 1.0, chunk=32)
    g1, g2 = torch.randn_like(lp), torch.randn_like(ent)
    (lp * g1 + ent * g2).sum().backward()
    hf, Wf = h.detach().float().requires_grad_(), W.detach().float().requires_grad_()
    lr, er = logprob_ref(hf, Wf, tgt, 1.0)
    (lr * g1 + er * g2).sum().backward()
    assert rel(h.grad, hf.grad) < 3e-2 and rel(W.grad, Wf.grad) < 3e-2
    with torch.no_grad():
        it = torch.full((n,), 1.0, device=DEV)
        seeds = torch.arange(n, device=DEV, dtype=torch.int64)
        posn = torch.arange(n, device=DEV, dtype=torch.int32)
        tok, slp = sample_from_hidden(h.detach(), W.detach(), it, seeds, posn)
        lp2, _ = lm_head_logprob(h.detach(), W.detach(), tok, 1.0)
        assert torch.equal(slp, lp2)
        tok_g, _ = sample_from_hidden(h.detach(), W.detach(), torch.zeros(n, device=DEV), seeds, posn)
        ref_g = (h.detach().float() @ W.detach().float().t()).argmax(-1)
        assert (tok_g.long() == ref_g).float().mean() > 0.95


def test_policy_loss_gae_grpo():
    from miles_b200.ops.rl import (PolicyLossCfg, gae, gae_ref, grpo_advantages, policy_loss,
                                   policy_loss_ref)
    torch.manual_seed(8)
    n = 5000
    lp = (torch.randn(n, device=DEV) * 0.3 - 1).requires_grad_()
    old = lp.detach() + torch.randn(n, device=DEV) * 0.2
    roll = old + torch.randn(n, device=DEV) * 0.2
    ref = old + torch.randn(n, device=DEV) * 0.1
    adv = torch.randn(n, device=DEV)
    wgt = torch.rand(n, device=DEV) / n
    cfg = PolicyLossCfg(0.2, 0.28, 3.0, True, 0.0, 2.0, 0.05, "low_var_kl")
    loss, m = policy_loss(lp, old, adv, wgt, cfg, roll, ref)
    loss.backward()
    lp2 = lp.detach().double().requires_grad_()
    lr, mr = policy_loss_ref(lp2, old.double(), adv.double(), wgt.double(), cfg, roll.double(), ref.double())
    lr.backward()
    assert abs(loss.item() - lr.item()) < 1e-4 * max(1, abs(lr.item()))
    assert (lp.grad.double() - lp2.grad).abs().max().item() < 1e-6
    rw = torch.randn(300, device=DEV)
    vals = torch.randn(300, device=DEV)
    cu = [0, 100, 101, 300]
    a, r = gae(rw, vals, cu, 0.99, 0.95)
    ar, rr = gae_ref(rw.cpu().double(), vals.cpu().double(), cu, 0.99, 0.95)
    assert (a.cpu().double() - ar).abs().max() < 1e-4
    rewards = (torch.rand(64, device=DEV) > 0.5).float()
    ga = grpo_advantages(rewards, 8)
    g = rewards.view(-1, 8)
    gr = ((g - g.mean(-1, keepdim=True)) / (g.std(-1, keepdim=True) + 1e-6)).view(-1)
    assert (ga - gr).abs().max() < 1e-4


def test_adam():
    from miles_b200.ops.optim import adam_, sqnorm_
    torch.manual_seed(9)
    n = 10000
    master = torch.randn(n, device=DEV)
    p = master.to(BF)
    g = torch.randn(n, device=DEV)
    m = torch.zeros(n, device=DEV)
    v = torch.zeros(n, device=DEV)
    sq = torch.zeros(1, device=DEV)
    sqnorm_(g, sq)
    assert abs(sq.item() - g.pow(2).sum().item()) / g.pow(2).sum().item() < 1e-5
    wref = master.clone()
    adam_(p, g, m, v, master=master, lr=1e-3, weight_decay=0.1, step=1, sqnorm=sq, max_norm=1.0)
    coef = min(1.0, 1.0 / (sq.sqrt().item() + 1e-6))
    gg = g * coef
    mref = 0.1 * gg
    vref = 0.001 * gg * gg
    upd = (mref / 0.1) / ((vref / 0.001).sqrt() + 1e-8)
    wref = wref - 1e-3 * (upd + 0.1 * wref)
    assert (master - wref).abs().max().item() < 1e-5
    assert torch.equal(p, master.to(BF))


@pytest.mark.parametrize("score_fn,T", [("softmax", 1), ("softmax", 64), ("sigmoid", 300)])
def test_fused_route_dispatch_matches_multi_kernel(score_fn, T):
    """The single-kernel decode route+dispatch equals router_fwd + permute plan + gather."""
    from miles_b200.ops._lib import lib
    from miles_b200.ops.moe import MoEPlan, RouterCfg

    torch.manual_seed(11)
    E, k, H = 128, 8, 2048
    cfg = RouterCfg(E, k, score_fn, True, 8 if score_fn == "sigmoid" else 1,
                    4 if score_fn == "sigmoid" else 1, 2.5 if score_fn == "sigmoid" else 1.0)
    logits = torch.randn(T, E, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1 if score_fn == "sigmoid" else None
    x = torch.randn(T, H, device=DEV, dtype=BF)
    idx = torch.empty(T, k, dtype=torch.int32, device=DEV)
    w = torch.empty(T, k, dtype=torch.float32, device=DEV)
    lib().router_fwd(logits, bias, None, idx, w, k, cfg.score_fn, cfg.renorm, cfg.n_group,
                     cfg.topk_group, cfg.scale)
    ref = MoEPlan(idx, E)
    xs_ref = ref.gather(x, zero_pad=False)
    plan, idx2, w2, xs = MoEPlan.fused(logits, bias, None, x, cfg)
    torch.cuda.synchronize()
    assert torch.equal(idx, idx2) and torch.equal(w, w2)
    assert torch.equal(ref.counts, plan.counts) and torch.equal(ref.offsets, plan.offsets)
    assert torch.equal(ref.dest, plan.dest)
    rows = ref.dest.long()
    assert torch.equal(xs[rows], xs_ref[rows])


def test_moe_layer_bf16_router_bias_matches_reference():
    """A routing bias stored in bf16 (a model parameter) is widened to fp32 before the router
    kernels read it: the layer's routing equals the fp32 reference's."""
    from miles_b200.ops.moe import RouterCfg, moe_experts, route_ref

    torch.manual_seed(3)
    T, H, E, k, F = 64, 256, 16, 4, 128
    x = torch.randn(T, H, device=DEV, dtype=torch.bfloat16)
    wr = (torch.randn(E, H, device=DEV) * 0.05).to(torch.bfloat16)
    w1 = (torch.randn(E, 2 * F, H, device=DEV) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E, H, F, device=DEV) * 0.05).to(torch.bfloat16)
    bias = (torch.randn(E, device=DEV) * 0.5).to(torch.bfloat16)
    cfg = RouterCfg(E, k, score_fn="sigmoid", renorm=True, n_group=4, topk_group=2, scale=1.0)
    got = []
    with torch.no_grad():
        moe_experts(x, wr, w1, w2, cfg, bias, None, got.append)
    logits = x.float() @ wr.float().t()
    ref, _ = route_ref(logits, cfg, bias)
    assert torch.equal(got[0].sort(1).values, ref.int().sort(1).values)
