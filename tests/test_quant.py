"""Quantizers: kernels vs PyTorch references (GPU) and round-trip error bounds (CPU)."""
import pytest
import torch

from miles_b200.ops import quant as Q


def test_refs_roundtrip_cpu():
    torch.manual_seed(0)
    w = torch.randn(300, 520)
    q, s = Q.fp8_block_quant(w)
    assert s.shape == (3, 5)
    err = (Q.fp8_block_dequant(q, s, dtype=torch.float32) - w).abs().max() / w.abs().max()
    assert err < 0.07
    q, s, z = Q.int4_fake_quant(w[:, :512], 128, True)
    assert (Q.int4_dequant(q, s, z, 128, True) - w[:, :512]).abs().max() / w.abs().max() < 0.2
    q, s, z = Q.int4_fake_quant(w[:, :512], 128, False)
    assert (Q.int4_dequant(q, s, z, 128, False) - w[:, :512]).abs().max() / w.abs().max() < 0.2
    p, bs, gs = Q.nvfp4_quant(w[:, :512])
    assert (Q.nvfp4_dequant(p, bs, gs, torch.float32) - w[:, :512]).abs().mean() / w.abs().mean() < 0.2
    y, e = Q.mxfp8_quant(w[:, :512])
    assert (Q.mxfp8_dequant(y, e, torch.float32) - w[:, :512]).abs().max() / w.abs().max() < 0.07


def test_int4_all_zero_group_pinned_cpu():
    """The int4 fake quantiser's scale floor (1e-8) on an all-zero group: codes 0, zero-point 0,
    scale 1e-8, in both modes, so the group dequantises to exact zeros."""
    w = torch.randn(2, 256)
    w[0, :128] = 0
    for sym in (True, False):
        q, s, z = Q.int4_fake_quant_ref(w, 128, sym)
        assert torch.all(q[0, :128] == (0 if sym else z[0, 0]))
        assert float(s[0, 0]) == pytest.approx(1e-8) and float(z[0, 0]) == 0.0
        assert torch.all(Q.int4_dequant(q, s, z, 128, sym)[0, :128] == 0)


@pytest.mark.gpu
def test_kernels_match_refs():
    torch.manual_seed(1)
    w = torch.randn(300, 520, device="cuda").to(torch.bfloat16)
    for ue in (False, True):
        q, s = Q.fp8_block_quant(w, ue8m0=ue)
        qr, sr = Q.fp8_block_quant_ref(w, ue8m0=ue)
        assert torch.allclose(s, sr, rtol=1e-6)
        assert (q.float() - qr.float()).abs().max() <= 32  # at most 1 ulp of e4m3 at the top binade
        assert (q.float() != qr.float()).float().mean() < 0.01
    x = torch.randn(64, 512, device="cuda").to(torch.bfloat16)
    q, s = Q.fp8_group_quant(x)
    assert q.shape == x.shape and s.shape == (64, 4)
    w2 = w[:, :512].contiguous()
    for sym in (True, False):
        q, s, z = Q.int4_fake_quant(w2, 128, sym)
        qr, sr, zr = Q.int4_fake_quant_ref(w2, 128, sym)
        assert (q.float() != qr.float()).float().mean() < 0.01
        assert torch.allclose(s.float(), sr.float(), rtol=1e-2)
    p, bs, gs = Q.nvfp4_quant(w2)
    d = Q.nvfp4_dequant(p, bs, gs, torch.float32)
    assert (d - w2.float()).abs().mean() / w2.float().abs().mean() < 0.2
    y, e = Q.mxfp8_quant(w2)
    yr, er = Q.mxfp8_quant(w2.cpu())
    assert torch.equal(e.cpu(), er)
