"""Unified block-scaled fp8 (e4m3) GEMMs on the tcgen05 kernel (miles_b200/csrc/gemm_fp8_sm100.cu).

Recipe (the reference's `--fp8-format e4m3 --fp8-recipe blockwise`, and its rollout engines'
128 x 128 block fp8 weights): weights are quantised in 128 x 128 blocks with one fp32 scale
each (`Fp8Weight`), activations in 1 x 128 groups along K with one fp32 scale per row and
group. The GEMM applies both scales per 128-wide K block in fp32 and rounds the output to bf16.

    quant_act(x)                       -> (q uint8 [M, K], s fp32 [K/128, M])
    Fp8Weight.from_bf16(w)             -> e4m3 weight + [N/128, K/128] scales
    fp8_linear(x, w8)                  -> x @ dequant(w8).T, bf16 out (x quantised on the fly)
    fp8_experts(xs, w1_8, w2_8, plan, save_gu)  -> MoE expert form (SwiGLU + down)
    register_fp8(w, w8) / fp8_of(w)    -> the fp8 copy that G.linear / the MoE layer use for w
    fp8_gemm_ref(...)                  -> fp32 PyTorch reference of the same math (tests)

Reference: examples/low_precision/README.md:17-18 (blockwise recipe),
miles/backends/megatron_utils/megatron_to_hf/processors/quantizer_fp8.py:10-109 (128 x 128
weight blocks with fp32 scale_inv).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from miles_b200.ops._lib import err_word, lib, use_native

FP8_MAX = 448.0


def quant_act_ref(x: torch.Tensor):
    """PyTorch form of the 1 x 128 activation quantisation (scale = amax / 448, amax floored at
    1e-12, q = saturate(x / scale)); returns (q e4m3 [M, K], s fp32 [K/128, M])."""
    M, K = x.shape
    xf = x.float().view(M, K // 128, 128)
    amax = xf.abs().amax(-1).clamp_min(1e-12)
    s = amax / FP8_MAX
    q = (xf * (1.0 / s)[..., None]).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(M, K)
    return q, s.t().contiguous()


def quant_act(x: torch.Tensor, offsets: torch.Tensor | None = None,
              counts: torch.Tensor | None = None):
    """x bf16 [M, K] -> (q uint8 [M, K] holding e4m3 bits, s fp32 [K/128, M]). For an
    expert-sorted buffer, `offsets` / `counts` limit the work to the rows that hold tokens (the
    other rows' q / s are left unwritten; their GEMM outputs are never stored)."""
    M, K = x.shape
    if K % 128:
        raise ValueError(f"fp8 activation quantisation needs K % 128 == 0 (K={K})")
    if not use_native(x):
        q, s = quant_act_ref(x)
        return q.view(torch.uint8), s
    q = torch.empty(M, K, dtype=torch.uint8, device=x.device)
    s = torch.empty(K // 128, M, dtype=torch.float32, device=x.device)
    lib().fp8_act_quant(x, q, s, offsets, counts)
    return q, s


@dataclass
class Fp8Weight:
    """A [N, K] weight (or E stacked [N, K] expert weights) in e4m3 with 128 x 128 block scales."""
    q: torch.Tensor  # uint8 [rows, K]
    s: torch.Tensor  # fp32 [rows/128, K/128]

    @staticmethod
    def empty_like(w: torch.Tensor) -> "Fp8Weight":
        """Buffers for w ([N, K], or [E, N, K] stored as E*N rows)."""
        K = w.shape[-1]
        rows = w.numel() // K
        if rows % 128 or K % 128:
            raise ValueError(f"fp8 weights need rows and K multiples of 128, got {tuple(w.shape)}")
        return Fp8Weight(torch.empty(rows, K, dtype=torch.uint8, device=w.device),
                         torch.empty(rows // 128, K // 128, dtype=torch.float32, device=w.device))

    @staticmethod
    def from_bf16(w: torch.Tensor) -> "Fp8Weight":
        w8 = Fp8Weight.empty_like(w)
        w8.requant_(w)
        return w8

    def requant_(self, w: torch.Tensor) -> None:
        """Re-quantise a new bf16 value into the same buffers (refit): the buffers keep their
        addresses, so decode graphs that read them stay valid."""
        w2 = w.reshape(self.q.shape)
        if use_native(w2):
            lib().fp8_block_cast(w2.contiguous(), 128, 128, self.q.view(torch.float8_e4m3fn), self.s, False)
            return
        from miles_b200.ops.quant import fp8_block_quant_ref

        q, s = fp8_block_quant_ref(w2, (128, 128))
        self.q.copy_(q.view(torch.uint8))
        self.s.copy_(s.float())

    def dequant(self) -> torch.Tensor:
        rows, K = self.q.shape
        w = self.q.view(torch.float8_e4m3fn).float().view(rows // 128, 128, K // 128, 128)
        return (w * self.s[:, None, :, None]).view(rows, K)


# fp8 copies of bf16 weights, keyed by the weight's storage address and shape: when a weight
# has one, G.linear / G.linear_swiglu / the MoE layer run the fp8 GEMM on it (forward), and the
# backward uses the bf16 weight.
_SHADOW: dict[int, tuple] = {}


def register_fp8(w: torch.Tensor, w8: Fp8Weight) -> None:
    _SHADOW[w.data_ptr()] = (tuple(w.shape), w8)


def unregister_fp8(w: torch.Tensor) -> None:
    _SHADOW.pop(w.data_ptr(), None)


def fp8_of(w: torch.Tensor) -> Fp8Weight | None:
    if not _SHADOW:
        return None
    e = _SHADOW.get(w.data_ptr())
    return e[1] if e is not None and e[0] == tuple(w.shape) else None


_SMS: dict[int, int] = {}


def _pick_bn(M: int, N: int, dev: torch.device) -> int:
    """Widest N tile (128, 64, 32) whose tile count fills at least half the machine; the
    narrowest otherwise. The tile width does not change the arithmetic."""
    i = dev.index or 0
    if i not in _SMS:
        _SMS[i] = torch.cuda.get_device_properties(dev).multi_processor_count
    sms = _SMS[i]
    mt = (M + 127) // 128
    for bn in (128, 64, 32):
        if mt * ((N + bn - 1) // bn) >= sms // 2 or bn == 32:
            return bn
    return 32


def fp8_gemm(aq, sa, w: Fp8Weight, out: torch.Tensor, M: int, N: int, *, mode: int = 0,
             group_offsets=None, group_counts=None, num_groups: int = 1, b_rows_per_group: int = 0,
             swiglu_f: int = 0, gu: torch.Tensor | None = None, bn: int | None = None):
    """Raw launcher (see mb_gemm_fp8)."""
    K = aq.shape[1]
    if bn is None:
        bn = _pick_bn(M if mode == 0 else aq.shape[0], N, aq.device)
        if swiglu_f:
            bn = max(bn, 64)
    lib().gemm_fp8(aq, sa, w.q, w.s, out, gu, M, N, K, mode, group_offsets, group_counts,
                   num_groups, b_rows_per_group, 4 if swiglu_f else 0, swiglu_f, bn,
                   err_word(aq.device))
    return out


def fp8_gemm_ref(aq, sa, w: Fp8Weight, M: int, N: int) -> torch.Tensor:
    """fp32 reference: dequantised operands, plain matmul (dense form)."""
    a = aq[:M].view(torch.float8_e4m3fn).float()
    K = a.shape[1]
    a = (a.view(M, K // 128, 128) * sa[:, :M].t()[..., None]).view(M, K)
    return a @ w.dequant()[:N].t()


def fp8_linear(x: torch.Tensor, w: Fp8Weight, out: torch.Tensor | None = None) -> torch.Tensor:
    """x [M, K] bf16 @ dequant(w).T -> bf16 [M, N]; x is quantised 1 x 128 on the fly."""
    M, K = x.shape
    N = w.q.shape[0]
    if not use_native(x):
        q, s = quant_act_ref(x)
        return fp8_gemm_ref(q.view(torch.uint8), s, w, M, N).to(x.dtype)
    xq, xs = quant_act(x)
    out = out if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    return fp8_gemm(xq, xs, w, out, M, N)


def fp8_gemm_grouped_ref(aq, sa, w: Fp8Weight, offsets, counts, n: int, swiglu_f: int = 0,
                         out_dtype=torch.bfloat16):
    """PyTorch form of the grouped fp8 GEMM (CPU runs and tests): per expert segment, the
    dequantised rows times the expert's dequantised weight, rounded to bf16 (SwiGLU applied with
    the kernel's rounding points when swiglu_f > 0). Padding rows are zero."""
    R, K = aq.shape
    a = aq.view(torch.float8_e4m3fn).float().view(R, K // 128, 128) * sa.t()[:R, :, None]
    a = a.view(R, K)
    E = offsets.numel() - 1
    wd = w.dequant().view(E, n, K)
    out = torch.zeros(R, swiglu_f if swiglu_f else n, dtype=out_dtype, device=aq.device)
    gu = torch.zeros(R, n, dtype=out_dtype, device=aq.device) if swiglu_f else None
    offs, cnt = offsets.tolist(), counts.tolist()
    for e in range(E):
        r0, c = offs[e], cnt[e]
        if c == 0:
            continue
        y = (a[r0:r0 + c] @ wd[e].t()).to(out_dtype)
        if swiglu_f:
            gu[r0:r0 + c] = y
            g, u = y[:, :swiglu_f].float(), y[:, swiglu_f:].float()
            out[r0:r0 + c] = ((g / (1 + torch.exp(-g))).to(out_dtype).float() * u).to(out_dtype)
        else:
            out[r0:r0 + c] = y
    return out, gu


def fp8_experts(xs: torch.Tensor, w1: Fp8Weight, w2: Fp8Weight, offsets: torch.Tensor,
                counts: torch.Tensor, E: int, F: int, H: int, save_gu: bool):
    """Routed-expert forward in fp8 over an expert-sorted buffer xs [R, H]: gate/up GEMM with
    the SwiGLU fused, 1 x 128 re-quantisation of its output, down GEMM. Returns (gu or None,
    a [R, F] bf16, ys [R, H] bf16), the tensors the bf16 path returns. Without a backward the
    padding rows are neither quantised nor stored."""
    R = xs.shape[0]
    cnt = None if save_gu else counts
    if not use_native(xs):
        xq, xsc = quant_act(xs)
        a, gu = fp8_gemm_grouped_ref(xq, xsc, w1, offsets, counts, 2 * F, swiglu_f=F, out_dtype=xs.dtype)
        aq, asc = quant_act(a)
        ys, _ = fp8_gemm_grouped_ref(aq, asc, w2, offsets, counts, H, out_dtype=xs.dtype)
        return (gu if save_gu else None), a, ys
    xq, xsc = quant_act(xs, offsets, cnt)
    a = torch.empty(R, F, dtype=torch.bfloat16, device=xs.device)
    gu = torch.empty(R, 2 * F, dtype=torch.bfloat16, device=xs.device) if save_gu else None
    fp8_gemm(xq, xsc, w1, a, R, 2 * F, mode=1, group_offsets=offsets, group_counts=cnt,
             num_groups=E, b_rows_per_group=2 * F, swiglu_f=F, gu=gu)
    aq, asc = quant_act(a, offsets, cnt)
    ys = torch.empty(R, H, dtype=torch.bfloat16, device=xs.device)
    fp8_gemm(aq, asc, w2, ys, R, H, mode=1, group_offsets=offsets, group_counts=cnt,
             num_groups=E, b_rows_per_group=H)
    return gu, a, ys
