"""Vocabulary-parallel log-prob kernels (csrc/rl_ops.cu logprob_part_kernel /
logprob_combine_kernel) on one GPU, with the TP ranks' vocabulary slices emulated as column
slices of one logit matrix: the combined log-prob / entropy match a plain fp32 PyTorch
log-softmax, one slice reproduces the single-GPU log-prob kernel bit for bit, and the slice-wise
backward (global lse, slice-relative targets) equals the full-vocabulary backward bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world,V", [(1, 4096), (2, 151936), (4, 32000), (8, 163840)])
def test_vocab_parallel_parts_combine(world, V):
    from miles_b200.ops._lib import lib

    torch.manual_seed(world)
    n = 67
    z = torch.randn(n, V, device="cuda") * 3
    t = torch.randint(0, V, (n,), device="cuda", dtype=torch.int32)
    inv_t = 1.0 / 0.7
    Vs = V // world
    parts = torch.empty(world, 4, n, device="cuda")
    for r in range(world):
        lo = r * Vs
        hi = V if r == world - 1 else lo + Vs
        lib().logprob_part(z[:, lo:hi], t, lo, inv_t, parts[r])
    lp, ent, lse = (torch.empty(n, device="cuda") for _ in range(3))
    lib().logprob_combine(parts, world, lp, ent, lse)
    lsm = (z * inv_t).log_softmax(-1)
    assert torch.allclose(lp, lsm.gather(1, t.long()[:, None])[:, 0], atol=2e-4, rtol=1e-5)
    assert torch.allclose(ent, -(lsm.exp() * lsm).sum(-1), atol=2e-4, rtol=1e-5)
    if world == 1:
        lp1, ent1, lse1 = (torch.empty(n, device="cuda") for _ in range(3))
        lib().logprob_fwd(z, t, inv_t, lp1, ent1, lse1)
        assert torch.equal(lp, lp1) and torch.equal(ent, ent1) and torch.equal(lse, lse1)
    # backward: slices with the global statistics equal the full-vocabulary kernel
    g_lp = torch.randn(n, device="cuda")
    g_ent = torch.randn(n, device="cuda")
    full = torch.empty(n, V, dtype=torch.bfloat16, device="cuda")
    lib().logprob_bwd(z, t, inv_t, lse, g_lp, g_ent, ent, full)
    sl = torch.empty_like(full)
    for r in range(world):
        lo = r * Vs
        hi = V if r == world - 1 else lo + Vs
        lib().logprob_bwd(z[:, lo:hi], (t - lo).int(), inv_t, lse, g_lp, g_ent, ent, sl[:, lo:hi])
    assert torch.equal(full, sl)
