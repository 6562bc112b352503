"""bf16 GEMMs on the tcgen05 kernel (miles_b200/csrc/gemm_sm100.cu).

`linear(x, w)` computes x @ w.T with an autograd backward that issues the data-grad as a
(K-major, MN-major) product and the weight-grad as an (MN-major, MN-major) product, so no
transposed copies are ever materialised. `grouped_linear` is the MoE expert form over tokens
sorted by expert with 128-row padded segments.

Reference roles replaced: TE linear layers (megatron_utils/model_provider.py:146-183),
TEGroupedLinear (--moe-grouped-gemm) and fsdp_utils/kernels/fused_experts.py:15-170.
"""
from __future__ import annotations

import torch

from miles_b200.ops._lib import err_word, lib, use_native

EPI_STORE_BF16, EPI_STORE_F32, EPI_ACC_BF16, EPI_ACC_F32 = 0, 1, 2, 3
_NUM_SMS: dict[int, int] = {}


def _num_sms(dev: torch.device) -> int:
    i = dev.index or 0
    if i not in _NUM_SMS:
        _NUM_SMS[i] = torch.cuda.get_device_properties(dev).multi_processor_count
    return _NUM_SMS[i]


def _pick_bn(M: int, N: int, dev: torch.device, groups: int = 1, narrow: bool = False,
             mtiles: int | None = None) -> int:
    """N tile width. The width never changes the per-element reduction order, so the choice does
    not affect results. Problems with enough 256-wide tiles to fill the machine use 256; smaller
    ones use the narrowest tile that still fits in one wave (a small-M GEMM costs about one
    K-long UMMA chain per wave, so more CTAs stream the weights in parallel at no extra
    latency). Tiles narrower than 64 are built for K-major operands only (``narrow``).
    ``mtiles`` bounds the number of M tiles that hold rows (grouped GEMMs whose padded buffer is
    mostly empty)."""
    mt = mtiles if mtiles is not None else (M + 127) // 128 * groups
    sms = _num_sms(dev)
    if mt * ((N + 255) // 256) >= sms:
        # several waves: pick the width with the fewest column-rounds of work
        # (waves x width), i.e. the least wave-quantisation loss; 256 unless another is >5% better
        def cost(bn):
            return -(-mt * ((N + bn - 1) // bn) // sms) * bn
        best = 256
        for bn in (192, 128):
            if cost(bn) < 0.95 * cost(best):
                best = bn
        return best
    cands = (256, 128, 64, 32, 16) if narrow else (256, 128, 64)
    best = cands[0]
    for bn in cands:
        if mt * ((N + bn - 1) // bn) > sms:
            break
        best = bn
    return best


def gemm(a: torch.Tensor, a_mn: bool, b: torch.Tensor, b_mn: bool, out: torch.Tensor,
         M: int, N: int, K: int, *, mode: int = 0, group_offsets: torch.Tensor | None = None,
         num_groups: int = 1, b_rows_per_group: int = 0, c_group_stride: int = 0,
         epi: int = EPI_STORE_BF16, alpha: float = 1.0, bn: int | None = None,
         group_counts: torch.Tensor | None = None) -> torch.Tensor:
    """Raw launcher: out[M,N] (=|+=) alpha * A[M,K] @ B[N,K]^T with stored operand layouts."""
    if bn is None:
        bn = _pick_bn(M, N, a.device, num_groups if mode == 2 else 1,
                      narrow=not a_mn and not b_mn)
    lib().gemm(a, a_mn, b, b_mn, out, M, N, K, mode, group_offsets, num_groups,
               b_rows_per_group, c_group_stride, epi, alpha, bn, group_counts, err_word(a.device))
    return out


def matmul_nt(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16, accumulate: bool = False) -> torch.Tensor:
    """a[M,K] @ b[N,K]^T (both K-major)."""
    M, K = a.shape
    N = b.shape[0]
    if not use_native(a):
        r = (a.float() @ b.float().t())
        if out is None:
            return r.to(out_dtype)
        if accumulate:
            out.add_(r.to(out.dtype))
        else:
            out.copy_(r)
        return out
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    epi = (EPI_STORE_F32 if out.dtype == torch.float32 else EPI_STORE_BF16) | (2 if accumulate else 0)
    return gemm(a, False, b, False, out, M, N, K, epi=epi)


def matmul_nn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """a[M,K] @ b[K,N] (b stored row-major [K,N], i.e. MN-major)."""
    M, K = a.shape
    N = b.shape[1]
    if not use_native(a):
        r = a.float() @ b.float()
        return r.to(torch.bfloat16) if out is None else out.copy_(r)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    return gemm(a, False, b, True, out, M, N, K)


def matmul_tn(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
              accumulate: bool = False) -> torch.Tensor:
    """a[K,M]^T @ b[K,N]: the weight-grad product (both stored with the contraction outermost)."""
    K, M = a.shape
    N = b.shape[1]
    if not use_native(a):
        r = a.float().t() @ b.float()
        if out is None:
            return r.to(torch.bfloat16)
        if accumulate:
            out.add_(r.to(out.dtype))
        else:
            out.copy_(r)
        return out
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a.device)
    epi = (EPI_STORE_F32 if out.dtype == torch.float32 else EPI_STORE_BF16) | (2 if accumulate else 0)
    return gemm(a, True, b, True, out, M, N, K, epi=epi)


# Persistent gradient buffers of parameters, keyed by the parameter's storage address. Lookups
# by address (not by tensor attribute) survive activation-checkpoint recomputation, whose saved
# tensors come back as detached aliases without Python attributes.
_MAIN_GRADS: dict[int, torch.Tensor] = {}


def register_main_grad(param: torch.Tensor, grad: torch.Tensor) -> None:
    _MAIN_GRADS[param.data_ptr()] = grad


def clear_main_grads() -> None:
    _MAIN_GRADS.clear()


def main_grad_of(w: torch.Tensor) -> torch.Tensor | None:
    g = _MAIN_GRADS.get(w.data_ptr())
    if g is not None and g.shape == w.shape:
        return g
    return getattr(w, "main_grad", None)


def _accumulate_wgrad(w: torch.Tensor, dy2: torch.Tensor, x2: torch.Tensor) -> torch.Tensor | None:
    """Weight-grad dW = dy^T x. When the parameter has a persistent gradient buffer (the
    trainer's flat gradient bucket), accumulate into it in place and return None."""
    main = main_grad_of(w)
    if main is not None:
        matmul_tn(dy2, x2, out=main, accumulate=True)
        return None
    return matmul_tn(dy2, x2)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        shp = x.shape
        y = matmul_nt(x.reshape(-1, shp[-1]), w)
        # Save the input itself, not a reshaped view of it: saving a view of a grad-requiring
        # input crashed the CUDA autograd thread in this torch build.
        ctx.save_for_backward(x, w)
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        x2 = x.reshape(-1, x.shape[-1])
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = matmul_nn(dy2, w).view(x.shape)
        if ctx.needs_input_grad[1]:
            dw = _accumulate_wgrad(w, dy2, x2)
        return dx, dw


class _Fp8Linear(_Linear):
    """Forward on the weight's registered fp8 copy (block-scaled fp8 GEMM, x quantised 1 x 128
    on the fly); the backward of the bf16 linear (data-grad with the bf16 weight, weight-grad
    into the bf16 parameter's gradient)."""

    @staticmethod
    def forward(ctx, x, w, w8):
        from miles_b200.ops.fp8 import fp8_linear

        shp = x.shape
        y = fp8_linear(x.reshape(-1, shp[-1]).contiguous(), w8)
        ctx.save_for_backward(x, w)
        return y.view(*shp[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        if not use_native(dy):
            x, w = ctx.saved_tensors
            x2 = x.reshape(-1, x.shape[-1])
            dy2 = dy.reshape(-1, dy.shape[-1])
            dx = (dy2 @ w).view(x.shape) if ctx.needs_input_grad[0] else None
            dw = (dy2.t() @ x2) if ctx.needs_input_grad[1] else None
            return dx, dw, None
        dx, dw = _Linear.backward(ctx, dy)
        return dx, dw, None


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y = x @ w.T  (w: [out, in], bf16). A weight with a registered fp8 copy
    (miles_b200.ops.fp8.register_fp8) runs its forward in block-scaled fp8."""
    from miles_b200.ops.fp8 import fp8_of

    w8 = fp8_of(w)
    if w8 is not None:
        if not (torch.is_grad_enabled() and (x.requires_grad or w.requires_grad)):
            from miles_b200.ops.fp8 import fp8_linear

            shp = x.shape
            return fp8_linear(x.reshape(-1, shp[-1]).contiguous(), w8).view(*shp[:-1], w.shape[0])
        return _Fp8Linear.apply(x, w, w8)
    if not use_native(x):
        return torch.nn.functional.linear(x, w)
    return _Linear.apply(x, w)


# ------------------------------------------------------------------------------------------
# GEMM + SwiGLU (fused epilogue): a = silu(x @ w_gate^T) * (x @ w_up^T), w = [gate; up]
# ------------------------------------------------------------------------------------------
def _swiglu_bn(M: int, F: int, dev: torch.device, mtiles: int | None = None) -> int | None:
    bn = _pick_bn(M, 2 * F, dev, narrow=True, mtiles=mtiles)
    for cand in sorted({max(bn, 32), 32, 64, 128, 256}, key=lambda c: (c < max(bn, 32), c)):
        if F % (cand // 2) == 0:
            return cand
    return None


def gemm_swiglu(x: torch.Tensor, w2d: torch.Tensor, F: int, *, mode: int = 0,
                offsets: torch.Tensor | None = None, num_groups: int = 1, save_gu: bool = False,
                mtiles: int | None = None, counts: torch.Tensor | None = None):
    """Fused GEMM + SwiGLU on stored operands (x: [M, K]; w2d: [groups * 2F, K]). Returns
    (a [M, F], gu [M, 2F] or None). Bitwise equal to the GEMM followed by the SwiGLU kernel."""
    M, K = x.shape
    a = torch.empty(M, F, dtype=torch.bfloat16, device=x.device)
    gu = torch.empty(M, 2 * F, dtype=torch.bfloat16, device=x.device) if save_gu else None
    bn = _swiglu_bn(M, F, x.device, mtiles)
    if bn is None:
        raise ValueError(f"no N tile divides F={F}")
    lib().gemm_swiglu(x, w2d, a, gu, M, F, K, mode, offsets, num_groups, bn, counts,
                      err_word(x.device))
    return a, gu


class _LinearSwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        shp = x.shape
        a, gu = gemm_swiglu(x.reshape(-1, shp[-1]).contiguous(), w, w.shape[0] // 2, save_gu=True)
        ctx.save_for_backward(x, w, gu)
        return a.view(*shp[:-1], w.shape[0] // 2)

    @staticmethod
    def backward(ctx, da):
        x, w, gu = ctx.saved_tensors
        from miles_b200.ops.norm import swiglu_bwd_raw

        x2 = x.reshape(-1, x.shape[-1])
        dgu = swiglu_bwd_raw(gu, da.reshape(-1, da.shape[-1]).contiguous())
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = matmul_nn(dgu, w).view(x.shape)
        if ctx.needs_input_grad[1]:
            dw = _accumulate_wgrad(w, dgu, x2)
        return dx, dw


class _Fp8LinearSwiGLU(_LinearSwiGLU):
    """SwiGLU projection with its forward on the registered fp8 copy (SwiGLU fused into the fp8
    GEMM epilogue); backward of the bf16 form."""

    @staticmethod
    def forward(ctx, x, w, w8):
        shp = x.shape
        a, gu = _fp8_swiglu(x.reshape(-1, shp[-1]).contiguous(), w8, w.shape[0] // 2, True)
        ctx.save_for_backward(x, w, gu)
        return a.view(*shp[:-1], w.shape[0] // 2)

    @staticmethod
    def backward(ctx, da):
        if not use_native(da):
            from miles_b200.ops.norm import swiglu_bwd_raw

            x, w, gu = ctx.saved_tensors
            dgu = swiglu_bwd_raw(gu, da.reshape(-1, da.shape[-1]))
            x2 = x.reshape(-1, x.shape[-1])
            dx = (dgu @ w).view(x.shape) if ctx.needs_input_grad[0] else None
            dw = (dgu.t() @ x2) if ctx.needs_input_grad[1] else None
            return dx, dw, None
        dx, dw = _LinearSwiGLU.backward(ctx, da)
        return dx, dw, None


def _fp8_swiglu(x2: torch.Tensor, w8, F: int, save_gu: bool):
    from miles_b200.ops import fp8 as F8

    M = x2.shape[0]
    if not use_native(x2):
        q, s = F8.quant_act(x2)
        offs = torch.tensor([0, M], dtype=torch.int32)
        cnt = torch.tensor([M], dtype=torch.int32)
        a, gu = F8.fp8_gemm_grouped_ref(q, s, w8, offs, cnt, 2 * F, swiglu_f=F, out_dtype=x2.dtype)
        return a, (gu if save_gu else None)
    q, s = F8.quant_act(x2)
    a = torch.empty(M, F, dtype=torch.bfloat16, device=x2.device)
    gu = torch.empty(M, 2 * F, dtype=torch.bfloat16, device=x2.device) if save_gu else None
    F8.fp8_gemm(q, s, w8, a, M, 2 * F, swiglu_f=F, gu=gu)
    return a, gu


def linear_swiglu(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """swiglu(x @ w.T) with w = [gate; up] ([2F, in]); one kernel on the GPU."""
    from miles_b200.ops.fp8 import fp8_of

    w8 = fp8_of(w)
    if w8 is not None:
        if not (torch.is_grad_enabled() and (x.requires_grad or w.requires_grad)):
            shp = x.shape
            a, _ = _fp8_swiglu(x.reshape(-1, shp[-1]).contiguous(), w8, w.shape[0] // 2, False)
            return a.view(*shp[:-1], w.shape[0] // 2)
        return _Fp8LinearSwiGLU.apply(x, w, w8)
    if not use_native(x):
        from miles_b200.ops.norm import swiglu_ref

        return swiglu_ref(torch.nn.functional.linear(x, w))
    if not (torch.is_grad_enabled() and (x.requires_grad or w.requires_grad)):
        shp = x.shape
        a, _ = gemm_swiglu(x.reshape(-1, shp[-1]).contiguous(), w, w.shape[0] // 2)
        return a.view(*shp[:-1], w.shape[0] // 2)
    return _LinearSwiGLU.apply(x, w)


# ------------------------------------------------------------------------------------------
# Grouped (MoE) GEMMs
# ------------------------------------------------------------------------------------------
def grouped_nt_swiglu(x: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor,
                      n_rows: int | None = None, save_gu: bool = False,
                      counts: torch.Tensor | None = None):
    """Per-expert swiglu(x_e @ w[e]^T) with w: [E, 2F, K] ([gate; up] per expert). Returns
    (a [R, F], gu [R, 2F] or None). With ``counts`` (rows per expert before padding) the
    padding rows of the outputs are left unwritten."""
    R, K = x.shape
    E, N2, _ = w.shape
    F = N2 // 2
    if not use_native(x):
        from miles_b200.ops.norm import swiglu_ref

        gu = grouped_nt(x, w, offsets)
        return swiglu_ref(gu), (gu if save_gu else None)
    return gemm_swiglu(x, w.view(E * N2, K), F, mode=1, offsets=offsets, num_groups=E,
                       save_gu=save_gu, mtiles=_grouped_mtiles(R, E, n_rows), counts=counts)


def _grouped_mtiles(R: int, E: int, n_rows: int | None) -> int:
    mt = (R + 127) // 128
    if n_rows is None:
        return mt
    return min(mt, (n_rows + 127) // 128 + min(E, n_rows))


def grouped_nt(x: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor,
               out: torch.Tensor | None = None, n_rows: int | None = None,
               counts: torch.Tensor | None = None) -> torch.Tensor:
    """Per-expert x_e @ w[e]^T. x: [R, K] sorted by expert with segments padded to 128 rows
    (offsets: int32 [E+1], device); w: [E, N, K]. Returns [R, N]. ``n_rows`` (the unpadded row
    count, if known) bounds the number of M tiles that hold rows."""
    R, K = x.shape
    E, N, _ = w.shape
    if out is None:
        out = torch.empty(R, N, dtype=torch.bfloat16, device=x.device)
    if not use_native(x):
        off = offsets.tolist()
        for e in range(E):
            a, b = off[e], off[e + 1]
            if b > a:
                out[a:b] = (x[a:b].float() @ w[e].float().t()).to(out.dtype)
        return out
    return gemm(x, False, w.view(E * N, K), False, out, R, N, K, mode=1, group_offsets=offsets,
                num_groups=E, b_rows_per_group=N,
                bn=_pick_bn(R, N, x.device, narrow=True, mtiles=_grouped_mtiles(R, E, n_rows)),
                group_counts=counts)


def grouped_nn(dy: torch.Tensor, w: torch.Tensor, offsets: torch.Tensor,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """Per-expert dy_e @ w[e] (data-grad). dy: [R, N]; w: [E, N, K]. Returns [R, K]."""
    R, N = dy.shape
    E, _, K = w.shape
    if out is None:
        out = torch.empty(R, K, dtype=torch.bfloat16, device=dy.device)
    if not use_native(dy):
        off = offsets.tolist()
        for e in range(E):
            a, b = off[e], off[e + 1]
            if b > a:
                out[a:b] = (dy[a:b].float() @ w[e].float()).to(out.dtype)
        return out
    return gemm(dy, False, w.view(E * N, K), True, out, R, K, N, mode=1, group_offsets=offsets,
                num_groups=E, b_rows_per_group=N, bn=_pick_bn(R, K, dy.device))


def grouped_tn(dy: torch.Tensor, x: torch.Tensor, offsets: torch.Tensor, E: int,
               out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """Per-expert dy_e^T @ x_e (weight-grad). dy: [R, N]; x: [R, K]. Returns [E, N, K]."""
    R, N = dy.shape
    K = x.shape[1]
    if out is None:
        out = torch.empty(E, N, K, dtype=torch.bfloat16, device=dy.device)
        accumulate = False
    if not use_native(dy):
        off = offsets.tolist()
        for e in range(E):
            a, b = off[e], off[e + 1]
            r = dy[a:b].float().t() @ x[a:b].float()
            if accumulate:
                out[e] += r.to(out.dtype)
            else:
                out[e] = r.to(out.dtype)
        return out
    epi = (EPI_STORE_F32 if out.dtype == torch.float32 else EPI_STORE_BF16) | (2 if accumulate else 0)
    return gemm(dy, True, x, True, out, N, K, R, mode=2, group_offsets=offsets, num_groups=E,
                c_group_stride=N * K, epi=epi)
