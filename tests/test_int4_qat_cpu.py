"""Int4 quantisation-aware training of the routed experts: the forward uses the fake-int4 expert
weights (equal to a model whose experts hold those values), the gradient reaches the bf16
weights straight through, and a weight-version change recomputes the fake-int4 values."""
import torch

from miles_b200.models.config import preset
from miles_b200.models.transformer import Transformer
from miles_b200.ops.attention import VarlenMeta
from miles_b200.ops.quant import int4_qat_weight


def test_int4_qat_forward_and_ste():
    cfg = preset("tiny-moe")
    tok = torch.randint(0, cfg.vocab_size, (50,), dtype=torch.int32)
    meta = VarlenMeta([0, 20, 50], "cpu")
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0, init_std=0.05)
    ref = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0, init_std=0.05)
    with torch.no_grad():
        for n, p in ref.params.items():
            if n.endswith(("experts.w1", "experts.w2")):
                p.copy_(int4_qat_weight(p.data, 128))
    m.enable_int4_qat(128)
    assert set(m.qat) == {n for n in m.params if n.endswith(("experts.w1", "experts.w2"))}
    h = m.forward_train(tok, meta)
    hr = ref.forward_train(tok, meta)
    assert torch.equal(h.detach(), hr.detach())
    h.square().mean().backward()
    hr.square().mean().backward()
    for n in m.qat:
        assert torch.allclose(m.params[n].grad, ref.params[n].grad, rtol=1e-5, atol=1e-7), n
    # the fake-int4 value is a fixed point and follows the weight version
    q = m.qat["layers.0.mlp.experts.w1"]
    assert torch.equal(int4_qat_weight(q, 128), q)
    before = q.clone()
    with torch.no_grad():
        m.params["layers.0.mlp.experts.w1"].mul_(3.0)
    m.sync_fp8()
    assert torch.equal(q, before)
    m.weight_version += 1
    m.sync_fp8()
    assert torch.allclose(q, before * 3.0, rtol=1e-6, atol=0)


def test_int4_qat_values():
    w = torch.randn(4, 256) * torch.tensor([1e-7, 1.0, 3.0, 0.0])[:, None]
    q = int4_qat_weight(w, 128)
    g = w.view(4, 2, 128)
    sc = (g.abs().amax(-1, keepdim=True) / 7).clamp_min(1e-5)
    levels = (q.view(4, 2, 128) / sc)
    assert torch.allclose(levels, levels.round(), atol=1e-4) and levels.abs().max() <= 7 + 1e-4
    assert torch.equal(q[3], torch.zeros(256))
