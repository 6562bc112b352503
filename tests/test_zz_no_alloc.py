"""Allocation-free decode attention entry point, called through its exported C symbol.

This entry point exists for callers that cannot allocate device memory themselves (code running
inside another framework's memory pool, or plain C/C++ hosts without a caching allocator): its
split-KV workspace is a fixed device array inside the library. The test checks that two calls
in a row match the regular entry point (which takes the workspace from its caller), and that a
request larger than the fixed workspace is refused. It lives in its own file so that pytest
collects it last.
"""
import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib():
    import miles_b200._C  # noqa: F401  (loads torch's shared libraries first)

    path = glob.glob(os.path.join(ROOT, "miles_b200", "_C*.so"))[0]
    lib = ctypes.CDLL(path)
    f = lib.mb_attn_decode_noalloc
    f.restype = ctypes.c_int
    # q, kc, vc, o, page_table, ctx_lens | B, max_pages | num_slots | nq, nkv | softmax_scale |
    # stream
    f.argtypes = ([ctypes.c_void_p] * 6 + [ctypes.c_int] * 2 + [ctypes.c_longlong]
                  + [ctypes.c_int] * 2 + [ctypes.c_float, ctypes.c_void_p])
    return f


def _err_fn():
    import miles_b200._C  # noqa: F401

    lib = ctypes.CDLL(glob.glob(os.path.join(ROOT, "miles_b200", "_C*.so"))[0])
    f = lib.mb_attn_decode_noalloc_error
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.c_void_p]
    return f


def _device_error() -> int:
    code = ctypes.c_int(-1)
    assert _err_fn()(ctypes.byref(code), torch.cuda.current_stream().cuda_stream) == 0
    return code.value


def _inputs(B, nq, nkv, lens, max_pages, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    slots = B * max_pages * 64
    kc = torch.randn(slots, nkv, 128, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(slots, nkv, 128, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(B, nq, 128, device="cuda", generator=g).to(torch.bfloat16)
    pt = torch.randperm(B * max_pages, device="cuda", generator=g).to(torch.int32).view(B, max_pages).contiguous()
    ctx = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, pt, ctx


def test_noalloc_matches_regular_entry_point():
    from miles_b200.ops.attention import decode_attention

    fn = _lib()
    B, nq, nkv, max_pages = 4, 32, 4, 40
    lens = [5, 1100, 2500, 64 * 40]
    q, kc, vc, pt, ctx = _inputs(B, nq, nkv, lens, max_pages)
    ref = decode_attention(q, kc, vc, pt, ctx)
    stream = torch.cuda.current_stream().cuda_stream
    scale = 1.0 / 128 ** 0.5
    for _ in range(2):  # two calls in a row share (and reuse) the fixed workspace
        out = torch.full_like(q, float("nan"))
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), pt.data_ptr(),
                ctx.data_ptr(), B, max_pages, kc.shape[0], nq, nkv, scale, stream)
        assert rc == 0
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max() / ref.float().abs().max()
        assert err < 2e-2
        assert torch.equal(out, ref)
        assert _device_error() == 0  # no bounded wait inside the kernels ran out


def test_noalloc_rejects_oversized_workspace():
    fn = _lib()
    B, nq, nkv, max_pages = 64, 64, 8, 160  # needs 64*64*10*130 floats > 1 Mi floats
    q, kc, vc, pt, ctx = _inputs(B, nq, nkv, [100] * B, max_pages)
    out = torch.zeros_like(q)
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), pt.data_ptr(), ctx.data_ptr(),
            B, max_pages, kc.shape[0], nq, nkv, 1.0, torch.cuda.current_stream().cuda_stream)
    assert rc == -9
