"""Optimizer-state offload around the rollout: parking the device-placed fp32 master and moments
in host buffers and bringing them back before the step leaves training bit-for-bit unchanged."""
import torch

from miles_b200.trainer.optimizer import FlatAdam


def _run(offload: bool):
    torch.manual_seed(0)
    p = torch.randn(4096)
    g = torch.zeros(4096)
    opt = FlatAdam(p, g, lr=1e-2, placement="device")
    for step in range(4):
        g.copy_(torch.randn(4096, generator=torch.Generator().manual_seed(step)))
        if offload:
            opt.offload(force=True)
            assert opt.m is None and opt.v is None and opt.master is None
        opt.step()
    return p.clone(), opt.state_dict()


def test_offload_roundtrip_is_exact():
    p0, s0 = _run(False)
    p1, s1 = _run(True)
    assert torch.equal(p0, p1)
    assert torch.equal(s0["m"], s1["m"]) and torch.equal(s0["v"], s1["v"])
    assert torch.equal(s0["master"], s1["master"])
