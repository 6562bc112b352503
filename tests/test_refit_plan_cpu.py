"""Peer-refit transfer plan (CPU): every byte / row of every parameter is covered exactly once,
no unit or bucket exceeds the staging capacity, fp8 units never split a 128-row block, and the
per-bucket owners' staging regions do not overlap."""
import os

import pytest
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")


@pytest.mark.parametrize("mode,cap,engines", [("bf16", 1 << 20, [1]), ("fp8", 1 << 20, [1, 2, 3]),
                                              ("fp8", 300 << 10, [1, 2]), ("bf16", 64 << 10, [1, 2, 3, 4])])
def test_refit_plan_covers_once(mode, cap, engines):
    from miles_b200.models.config import preset
    from miles_b200.models.transformer import Transformer
    from miles_b200.parallel.refit import refit_buckets, refit_units

    m = Transformer(preset("tiny-moe"), device="cpu", dtype=torch.bfloat16, materialize=False)
    units = refit_units(m, mode, cap)
    buckets = refit_buckets(units, engines, cap)
    covered = {}
    for b in buckets:
        regions = {e: [] for e in engines}
        for name, kind, lo, hi, owner, off in b:
            nb = next(u[4] for u in units if u[:4] == (name, kind, lo, hi))
            assert nb <= cap and off + nb <= cap
            regions[owner].append((off, off + nb))
            covered.setdefault((name, kind), []).append((lo, hi))
            if kind == "fp8":
                assert lo % 128 == 0
        for rs in regions.values():
            rs.sort()
            assert all(a[1] <= b_[0] for a, b_ in zip(rs, rs[1:]))
    for s in m.specs:
        p = m.params[s.name]
        keys = [k for k in covered if k[0] == s.name]
        assert len(keys) == 1, s.name
        kind = keys[0][1]
        total = (p.numel() // p.shape[-1] if kind == "fp8" else p.numel() * p.element_size())
        iv = sorted(covered[keys[0]])
        assert iv[0][0] == 0 and iv[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(iv, iv[1:]))
