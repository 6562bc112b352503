"""tcgen05 GEMM numerics against a PyTorch fp32 reference of the same product."""
import pytest
import torch

from miles_b200.ops import gemm as G

pytestmark = pytest.mark.gpu


def _ref(a, b):
    return a.float() @ b.float().t()


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err / scale < tol, f"rel err {err / scale}"


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 520, 200), (2048, 2048, 2048),
                                   (1, 4096, 2048), (64, 5120, 2048), (4096, 1536, 768)])
def test_nt(M, N, K):
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    _close(G.matmul_nt(a, b), _ref(a, b))
    torch.cuda.synchronize()
    from miles_b200.ops import check_device_error
    check_device_error()


@pytest.mark.parametrize("bn", [16, 32, 64, 128, 256])
def test_tile_width_invariance(bn):
    """Different N-tile widths give bitwise identical results (batch invariance)."""
    torch.manual_seed(1)
    a = torch.randn(256, 1024, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16)
    ref = G.gemm(a, False, b, False, torch.empty(256, 512, device="cuda", dtype=torch.bfloat16),
                 256, 512, 1024, bn=256)
    out = G.gemm(a, False, b, False, torch.empty(256, 512, device="cuda", dtype=torch.bfloat16),
                 256, 512, 1024, bn=bn)
    assert torch.equal(ref, out)
    # row 7 computed alone equals row 7 computed inside the batch
    one = G.matmul_nt(a[7:8].contiguous(), b)
    assert torch.equal(one[0], ref[7])
    # small-M GEMMs (short A boxes, narrow tiles) match the batched rows bitwise
    for m in (3, 8, 40, 64, 100):
        part = G.gemm(a[:m].contiguous(), False, b, False,
                      torch.empty(m, 512, device="cuda", dtype=torch.bfloat16), m, 512, 1024,
                      bn=bn)
        assert torch.equal(part, ref[:m]), m


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (1000, 2048, 768)])
def test_nn_and_tn(M, N, K):
    torch.manual_seed(2)
    dy = torch.randn(M, N, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    _close(G.matmul_nn(dy, w), dy.float() @ w.float())
    _close(G.matmul_tn(dy, x), dy.float().t() @ x.float())
    acc = torch.ones(N, K, device="cuda", dtype=torch.float32)
    G.matmul_tn(dy, x, out=acc, accumulate=True)
    _close(acc, dy.float().t() @ x.float() + 1)


def test_linear_autograd():
    torch.manual_seed(3)
    x = torch.randn(3, 100, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(768, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y = G.linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xr = x.detach().float().requires_grad_()
    wr = w.detach().float().requires_grad_()
    yr = xr @ wr.t()
    yr.backward(g.float())
    _close(y, yr)
    _close(x.grad, xr.grad)
    _close(w.grad, wr.grad)


def _grouped_inputs(E, counts, K, N):
    off = [0]
    for c in counts:
        off.append(off[-1] + (c + 127) // 128 * 128)
    R = off[-1] + 128
    x = torch.zeros(R, K, device="cuda", dtype=torch.bfloat16)
    for e, c in enumerate(counts):
        x[off[e]:off[e] + c] = torch.randn(c, K, device="cuda", dtype=torch.bfloat16)
    offs = torch.tensor(off, dtype=torch.int32, device="cuda")
    return x, offs, off


def test_grouped():
    torch.manual_seed(4)
    E, K, N = 8, 256, 384
    counts = [5, 0, 130, 256, 1, 77, 0, 300]
    x, offs, off = _grouped_inputs(E, counts, K, N)
    w = torch.randn(E, N, K, device="cuda", dtype=torch.bfloat16)
    y = G.grouped_nt(x, w, offs)
    dy = torch.zeros(x.shape[0], N, device="cuda", dtype=torch.bfloat16)
    for e, c in enumerate(counts):
        a = off[e]
        if c:
            _close(y[a:a + c], x[a:a + c].float() @ w[e].float().t())
        dy[a:a + c] = torch.randn(c, N, device="cuda", dtype=torch.bfloat16)
    dx = G.grouped_nn(dy, w, offs)
    dw = G.grouped_tn(dy, x, offs, E)
    for e, c in enumerate(counts):
        a = off[e]
        if c:
            _close(dx[a:a + c], dy[a:a + c].float() @ w[e].float())
        ref = dy[a:a + c].float().t() @ x[a:a + c].float()
        if c:
            _close(dw[e], ref)
        else:
            assert dw[e].abs().max().item() == 0


def test_worker_thread_and_error_path():
    """A kernel first used on the main thread also runs from a fresh thread (the autograd
    worker), and a rejected configuration raises instead of crashing."""
    import threading
    a = torch.randn(300, 768, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(768, 512, device="cuda", dtype=torch.bfloat16)
    ref = G.matmul_nn(a, w)
    out = {}
    t = threading.Thread(target=lambda: out.setdefault("y", G.matmul_nn(a, w)))
    t.start()
    t.join()
    assert torch.equal(out["y"], ref)
    with pytest.raises(RuntimeError):
        G.gemm(a, False, w, True, torch.empty(300, 512, device="cuda", dtype=torch.bfloat16),
               300, 512, 768, bn=96)


@pytest.mark.parametrize("M,F,K", [(1, 768, 2048), (64, 768, 2048), (300, 1024, 512),
                                   (2048, 9728 // 4, 640)])
def test_swiglu_epilogue_bitwise(M, F, K):
    """GEMM with the fused SwiGLU epilogue equals GEMM followed by the SwiGLU kernel, bit for
    bit, and matches the fp32 reference."""
    from miles_b200.ops.norm import swiglu, swiglu_ref

    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(2 * F, K, device="cuda", dtype=torch.bfloat16) * 0.05
    gu_ref = G.matmul_nt(x, w)
    a_ref = swiglu(gu_ref)
    a, gu = G.gemm_swiglu(x, w, F, save_gu=True)
    assert torch.equal(gu, gu_ref)
    assert torch.equal(a, a_ref)
    _close(a, swiglu_ref((x.float() @ w.float().t()).to(torch.bfloat16)).float())


def test_grouped_swiglu_bitwise():
    from miles_b200.ops.moe import MoEPlan
    from miles_b200.ops.norm import swiglu

    torch.manual_seed(4)
    E, F, K, T, k = 16, 256, 512, 40, 4
    idx = torch.stack([torch.randperm(E, device="cuda")[:k] for _ in range(T)]).int()
    plan = MoEPlan(idx, E)
    x = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
    xs = plan.gather(x)
    w = torch.randn(E, 2 * F, K, device="cuda", dtype=torch.bfloat16) * 0.05
    gu_ref = G.grouped_nt(xs, w, plan.offsets)
    a, gu = G.grouped_nt_swiglu(xs, w, plan.offsets, n_rows=T * k, save_gu=True)
    total = int(plan.offsets[-1])
    assert torch.equal(gu[:total], gu_ref[:total])
    assert torch.equal(a[:total], swiglu(gu_ref[:total]))
