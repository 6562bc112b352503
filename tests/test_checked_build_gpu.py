"""Checked build (miles_b200._C_checked, compiled with MB_CHECKS=1): bounds guards record an
error code in their unit's check word and skip the bad access instead of faulting; the regular
build's words stay zero. Small shapes, one bad index each."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _checked():
    try:
        import miles_b200._C  # noqa: F401  (torch libraries first)
        from miles_b200 import _C_checked
    except ImportError:
        pytest.skip("checked extension not built")
    return _C_checked


def test_moe_gather_guard_records_and_skips():
    ck = _checked()
    ck.check_words(True)
    x = torch.arange(2 * 64, device="cuda", dtype=torch.float32).view(2, 64).to(torch.bfloat16)
    xs = torch.zeros(16, 64, device="cuda", dtype=torch.bfloat16)
    dest = torch.tensor([3, 99], device="cuda", dtype=torch.int32)  # row 99 is outside xs
    assert ck.moe_gather(x, dest, 1, xs) == 0
    torch.cuda.synchronize()
    assert torch.equal(xs[3], x[0])                # the valid row was copied
    assert ck.check_words(True) == [41, 0]         # moe unit: destination row out of range
    assert ck.check_words(False) == [0, 0]         # cleared


def test_decode_prep_guard_records_and_skips():
    ck = _checked()
    from miles_b200 import _C

    S, P, B = 4, 3, 2
    i32 = dict(dtype=torch.int32, device="cuda")
    rows = torch.tensor([1, S + 7], **i32)        # second batch row names no slot
    args = [torch.zeros(S + 1, **i32), torch.full((S + 1,), 5, **i32), torch.zeros(S + 1, **i32),
            torch.zeros(S + 1, P, **i32), torch.ones(S + 1, device="cuda"),
            torch.zeros(S + 1, dtype=torch.int64, device="cuda")]
    outs = [torch.zeros(B, **i32), torch.zeros(B, **i32), torch.zeros(B, **i32),
            torch.zeros(B, dtype=torch.int64, device="cuda"), torch.zeros(B, P, **i32),
            torch.zeros(B, device="cuda"), torch.zeros(B, dtype=torch.int64, device="cuda")]
    ck.check_words(True)
    assert ck.decode_prep(rows, S, *args, *outs, None, S) == 0
    torch.cuda.synchronize()
    assert ck.check_words(True) == [0, 51]
    assert int(outs[1][0]) == 5                    # the valid row was prepared
    assert _C.check_words(False) == [0, 0]         # the regular build has no guards
