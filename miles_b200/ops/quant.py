"""Weight / activation quantizers (kernels in csrc/quant.cu) with PyTorch references.

    fp8_block_quant(w, block=(128,128), ue8m0=False) -> (w_fp8 e4m3, scale_inv fp32 [ceil(M/bm), ceil(N/bn)])
    fp8_group_quant(x, group=128)                    -> (x_fp8, scale fp32 [M, ceil(N/group)])
    int4_fake_quant(w, group=128, sym=True)          -> (q, scale, zero) in w's dtype
    nvfp4_quant(w)                                   -> (packed uint8 [M, N/2], block scale e4m3 [M, N/16], global fp32)
    mxfp8_quant(w)                                   -> (w_fp8, scale exponent uint8 [M, N/32])

Reference: utils/fp8_kernel.py (blockwise_cast_to_fp8_triton), kernels/int4_qat/*,
megatron_to_hf/processors/quantizer_{fp8,nvfp4,mxfp8,compressed_tensors}.py.
"""
from __future__ import annotations

import math

import torch

from miles_b200.ops._lib import lib, use_native

FP8_MAX = 448.0


def _ue8m0(s: torch.Tensor) -> torch.Tensor:
    return torch.pow(2.0, torch.ceil(torch.log2(s.clamp_min(1e-30))))


def fp8_block_quant_ref(w: torch.Tensor, block=(128, 128), ue8m0: bool = False):
    M, N = w.shape
    bm, bn = block
    gm, gn = math.ceil(M / bm), math.ceil(N / bn)
    pad = torch.zeros(gm * bm, gn * bn, dtype=torch.float32, device=w.device)
    pad[:M, :N] = w.float()
    blk = pad.view(gm, bm, gn, bn)
    amax = blk.abs().amax(dim=(1, 3)).clamp_min(1e-12)
    s = amax / FP8_MAX
    if ue8m0:
        s = _ue8m0(s)
    q = (blk / s[:, None, :, None]).clamp(-FP8_MAX, FP8_MAX).view(gm * bm, gn * bn)[:M, :N]
    return q.to(torch.float8_e4m3fn), s


def fp8_block_quant(w: torch.Tensor, block=(128, 128), ue8m0: bool = False):
    if not use_native(w):
        return fp8_block_quant_ref(w, block, ue8m0)
    w = w.contiguous().to(torch.bfloat16)
    M, N = w.shape
    y = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=w.device)
    s = torch.empty(math.ceil(M / block[0]), math.ceil(N / block[1]), dtype=torch.float32, device=w.device)
    lib().fp8_block_cast(w, block[0], block[1], y, s, ue8m0)
    return y, s


def fp8_block_dequant(q: torch.Tensor, s: torch.Tensor, block=(128, 128), dtype=torch.bfloat16):
    M, N = q.shape
    sf = s.repeat_interleave(block[0], 0)[:M].repeat_interleave(block[1], 1)[:, :N]
    return (q.float() * sf).to(dtype)


def fp8_group_quant(x: torch.Tensor, group: int = 128, ue8m0: bool = False):
    M, N = x.shape
    if not use_native(x):
        g = math.ceil(N / group)
        pad = torch.zeros(M, g * group, dtype=torch.float32, device=x.device)
        pad[:, :N] = x.float()
        s = pad.view(M, g, group).abs().amax(-1).clamp_min(1e-12) / FP8_MAX
        if ue8m0:
            s = _ue8m0(s)
        q = (pad.view(M, g, group) / s[..., None]).clamp(-FP8_MAX, FP8_MAX).view(M, -1)[:, :N]
        return q.to(torch.float8_e4m3fn), s
    x = x.contiguous().to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(M, math.ceil(N / group), dtype=torch.float32, device=x.device)
    lib().fp8_group_cast(x, group, y, s, ue8m0)
    return y, s


def int4_fake_quant_ref(w: torch.Tensor, group: int = 128, sym: bool = True):
    M, N = w.shape
    g = w.float().view(M, N // group, group)
    if sym:
        s = (g.abs().amax(-1) / 7).clamp_min(1e-8)
        q = torch.round(g / s[..., None]).clamp(-8, 7)
        z = torch.zeros_like(s)
    else:
        mx, mn = g.amax(-1), g.amin(-1)
        s = ((mx - mn) / 15).clamp_min(1e-8)
        z = torch.clamp(-torch.round(mn / s), 0, 15)
        q = torch.clamp(torch.round(g / s[..., None]) + z[..., None], 0, 15)
    return q.view(M, N).to(w.dtype), s.to(w.dtype), z.to(w.dtype)


def int4_fake_quant(w: torch.Tensor, group: int = 128, sym: bool = True):
    if not use_native(w):
        return int4_fake_quant_ref(w, group, sym)
    w = w.contiguous()
    M, N = w.shape
    q = torch.empty_like(w)
    s = torch.empty(M, N // group, dtype=w.dtype, device=w.device)
    z = torch.empty(M, N // group, dtype=w.dtype, device=w.device)
    lib().int4_fake_quant(w, group, sym, q, s, z)
    return q, s, z


@torch.no_grad()
def int4_qat_weight(w: torch.Tensor, group: int = 128, out: torch.Tensor | None = None,
                    rows_per_chunk: int = 1 << 16) -> torch.Tensor:
    """The value an int4 quantisation-aware-training forward uses for a weight: symmetric int4 in
    groups of `group` along the last dim, scale = max(|w| over the group / 7, 1e-5) in fp32,
    q = clamp(round(w / scale), -7, 7), result q * scale in the weight's dtype. Processed in row
    chunks (bounded fp32 temporaries). Reference: the fake-int4 STE of the grouped expert linear
    (docker/patch/latest/megatron.patch, _FakeInt4QuantizationSTE)."""
    K = w.shape[-1]
    if K % group:
        raise ValueError(f"int4 QAT needs the input dim ({K}) to be a multiple of {group}")
    w2 = w.reshape(-1, K)
    out = out if out is not None else torch.empty_like(w)
    o2 = out.view(-1, K)
    for a in range(0, w2.shape[0], rows_per_chunk):
        g = w2[a:a + rows_per_chunk].float().view(-1, K // group, group)
        sc = (g.abs().amax(-1, keepdim=True) / 7).clamp_min(1e-5)
        o2[a:a + rows_per_chunk] = (torch.round(g / sc).clamp(-7, 7) * sc).view(-1, K).to(w.dtype)
    return out


def int4_dequant(q, s, z, group: int = 128, sym: bool = True):
    M, N = q.shape
    qf = q.float().view(M, N // group, group)
    if sym:
        return (qf * s.float()[..., None]).view(M, N)
    return ((qf - z.float()[..., None]) * s.float()[..., None]).view(M, N)


_E2M1 = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6], dtype=torch.float32)


def nvfp4_quant(w: torch.Tensor):
    """Returns (packed uint8 [M, N/2], block scales e4m3 [M, N/16], global scale fp32)."""
    M, N = w.shape
    amax = w.float().abs().max().clamp_min(1e-12)
    gs = float(amax / (FP8_MAX * 6.0))
    if not use_native(w):
        g = w.float().view(M, N // 16, 16)
        bs = (g.abs().amax(-1) / 6.0 / gs).clamp(max=FP8_MAX).to(torch.float8_e4m3fn)
        s = bs.float() * gs
        v = torch.where(s[..., None] > 0, g / s[..., None], torch.zeros_like(g))
        table = _E2M1.to(w.device)
        mag = (v.abs()[..., None] - table).abs()
        # tie -> even code: prefer the lower index on equal distance when the lower is even
        code = mag.argmin(-1)
        code = torch.where((v < 0) & (code > 0), code + 8, code).to(torch.uint8).view(M, N)
        packed = (code[:, 0::2] | (code[:, 1::2] << 4)).contiguous()
        return packed, bs, gs
    w = w.contiguous().to(torch.bfloat16)
    packed = torch.empty(M, N // 2, dtype=torch.uint8, device=w.device)
    bs = torch.empty(M, N // 16, dtype=torch.float8_e4m3fn, device=w.device)
    lib().nvfp4_quant(w, gs, packed, bs)
    return packed, bs, gs


def nvfp4_dequant(packed, bs, gs, dtype=torch.bfloat16):
    M = packed.shape[0]
    lo, hi = packed & 0xF, packed >> 4
    codes = torch.stack([lo, hi], -1).view(M, -1).long()
    table = _E2M1.to(packed.device)
    vals = table[codes & 7] * torch.where(codes >= 8, -1.0, 1.0)
    s = bs.float().repeat_interleave(16, 1) * gs
    return (vals * s).to(dtype)


def mxfp8_quant(w: torch.Tensor):
    M, N = w.shape
    if not use_native(w):
        g = w.float().view(M, N // 32, 32)
        s = _ue8m0(g.abs().amax(-1).clamp_min(1e-30) / FP8_MAX)
        q = (g / s[..., None]).clamp(-FP8_MAX, FP8_MAX).view(M, N).to(torch.float8_e4m3fn)
        e = (torch.log2(s) + 127).round().to(torch.uint8)
        return q, e
    w = w.contiguous().to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.float8_e4m3fn, device=w.device)
    e = torch.empty(M, N // 32, dtype=torch.uint8, device=w.device)
    lib().mxfp8_quant(w, y, e)
    return y, e


def mxfp8_dequant(q, e, dtype=torch.bfloat16):
    s = torch.pow(2.0, e.float() - 127).repeat_interleave(32, 1)
    return (q.float() * s).to(dtype)
