"""RMSNorm, fused QK-norm + RoPE and SwiGLU (kernels in csrc/norm_rope_act.cu).

CPU tensors take a PyTorch reference path with the same rounding points as the kernels
(normalised value rounded to bf16 before the weight multiply, as in HF Qwen3RMSNorm).
"""
from __future__ import annotations

import math

import torch

from miles_b200.ops._lib import lib, use_native


# ------------------------------------------------------------------------------------------
# RMSNorm
# ------------------------------------------------------------------------------------------
def rms_norm_ref(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * (xf * r).to(x.dtype).float()).to(x.dtype)


def _nparts(rows: int) -> int:
    return max(1, min(296, (rows + 63) // 64))


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        xc = x.contiguous()
        y = torch.empty_like(xc)
        rows = xc.numel() // xc.shape[-1]
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        lib().rmsnorm_fwd(xc, None, w, None, y, rstd, eps)
        ctx.save_for_backward(xc, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch.empty_like(x)
        H = x.shape[-1]
        rows = x.numel() // H
        part = torch.empty(_nparts(rows), H, dtype=torch.float32, device=x.device)
        dwf = torch.empty(H, dtype=torch.float32, device=x.device)
        lib().rmsnorm_bwd(dy, x, w, rstd, None, dx, part, dwf, None, False)
        return dx, dwf.to(w.dtype), None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if not use_native(x):
        return rms_norm_ref(x, w, eps)
    return _RMSNorm.apply(x, w, eps)


class _AddRMSNorm(torch.autograd.Function):
    """h = x + res; y = rmsnorm(h). Returns (y, h)."""

    @staticmethod
    def forward(ctx, x, res, w, eps):
        x = x.contiguous()
        res = res.contiguous()
        h = torch.empty_like(x)
        y = torch.empty_like(x)
        rows = x.numel() // x.shape[-1]
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        lib().rmsnorm_fwd(x, res, w, h, y, rstd, eps)
        ctx.save_for_backward(h, w, rstd)
        return y, h

    @staticmethod
    def backward(ctx, dy, dh):
        h, w, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dy = dy.contiguous()
        dx = torch.empty_like(h)
        H = h.shape[-1]
        rows = h.numel() // H
        part = torch.empty(_nparts(rows), H, dtype=torch.float32, device=h.device)
        dwf = torch.empty(H, dtype=torch.float32, device=h.device)
        lib().rmsnorm_bwd(dy, h, w, rstd, dh.contiguous() if dh is not None else None, dx, part,
                          dwf, None, False)
        return dx, dx, dwf.to(w.dtype), None


def add_rms_norm(x: torch.Tensor, res: torch.Tensor, w: torch.Tensor, eps: float = 1e-6):
    """Fused residual add + RMSNorm: returns (norm(x + res), x + res)."""
    if not use_native(x):
        h = (x.float() + res.float()).to(x.dtype)
        return rms_norm_ref(h, w, eps), h
    return _AddRMSNorm.apply(x, res, w, eps)


# ------------------------------------------------------------------------------------------
# RoPE tables + fused QK-norm/RoPE
# ------------------------------------------------------------------------------------------
_ROPE_CACHE: dict = {}


def rope_tables(max_pos: int, head_dim: int, theta: float, device, scaling: dict | None = None):
    """cos/sin tables [max_pos, head_dim/2] fp32 (rotate-half convention). `scaling` accepts
    the HF rope_scaling dict for 'yarn' (DeepSeek/MLA), 'llama3' (Llama 3.1 frequency bands)
    and 'linear'."""
    key = (max_pos, head_dim, theta, str(device), repr(scaling))
    t = _ROPE_CACHE.get(key)
    if t is not None:
        return t
    half = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float64) * 2 / head_dim))
    mscale = 1.0
    if scaling:
        typ = scaling.get("rope_type", scaling.get("type"))
        factor = float(scaling.get("factor", 1.0))
        if typ == "linear":
            inv = inv / factor
        elif typ == "llama3":
            # long wavelengths divided by `factor`, short ones kept, a linear blend between
            orig = float(scaling.get("original_max_position_embeddings", 8192))
            lo, hi = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
            wavelen = 2 * math.pi / inv
            smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0, 1)
            inv = torch.where(wavelen < orig / hi, inv,
                              torch.where(wavelen > orig / lo, inv / factor,
                                          (1 - smooth) * inv / factor + smooth * inv))
        elif typ == "yarn":
            orig = float(scaling.get("original_max_position_embeddings", 4096))
            beta_fast = float(scaling.get("beta_fast", 32))
            beta_slow = float(scaling.get("beta_slow", 1))

            def corr(nrot):
                return (head_dim * math.log(orig / (nrot * 2 * math.pi))) / (2 * math.log(theta))

            low = max(math.floor(corr(beta_fast)), 0)
            high = min(math.ceil(corr(beta_slow)), half - 1)
            ramp = ((torch.arange(half, dtype=torch.float64) - low) / max(high - low, 1e-3)).clamp(0, 1)
            inv = inv / factor * ramp + inv * (1 - ramp)
            ms = float(scaling.get("mscale", 1.0))
            msa = float(scaling.get("mscale_all_dim", 0.0))

            def get_m(s, m):
                return 1.0 if s <= 1 else 0.1 * m * math.log(s) + 1.0

            mscale = get_m(factor, ms) / get_m(factor, msa) if msa else get_m(factor, ms)
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos[:, None] * inv[None, :]
    cos = (ang.cos() * mscale).float().to(device)
    sin = (ang.sin() * mscale).float().to(device)
    _ROPE_CACHE[key] = (cos, sin)
    return cos, sin


def qk_norm_rope_ref(qkv, qw, kw, pos, cos, sin, nq, nkv, eps, use_norm=True):
    T = qkv.shape[0]
    D = qkv.shape[1] // (nq + 2 * nkv)
    half = D // 2
    x = qkv.view(T, nq + 2 * nkv, D)
    q, k, v = x[:, :nq], x[:, nq:nq + nkv], x[:, nq + nkv:]

    def norm(t, w):
        if not use_norm:
            return t.float()
        tf = t.float()
        r = torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + eps)
        return ((tf * r).to(qkv.dtype).float() * w.float()).to(qkv.dtype).float()

    def rope(t):
        c = cos[pos.long()][:, None, :]
        s = sin[pos.long()][:, None, :]
        a, b = t[..., :half], t[..., half:]
        return torch.cat([a * c - b * s, b * c + a * s], -1).to(qkv.dtype)

    return rope(norm(q, qw)), rope(norm(k, kw)), v.contiguous()


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, qw, kw, pos, cos, sin, nq, nkv, eps, use_norm):
        T = qkv.shape[0]
        dev = qkv.device
        q = torch.empty(T, nq, 128, dtype=torch.bfloat16, device=dev)
        k = torch.empty(T, nkv, 128, dtype=torch.bfloat16, device=dev)
        v = torch.empty(T, nkv, 128, dtype=torch.bfloat16, device=dev)
        rstd = torch.empty(T, nq + nkv, dtype=torch.float32, device=dev) if use_norm else None
        lib().qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, q, k, v, None, nkv * 128, rstd, nq, nkv,
                               eps, use_norm)
        ctx.save_for_backward(qkv, qw, kw, pos, cos, sin, rstd)
        ctx.cfg = (nq, nkv, use_norm)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, qw, kw, pos, cos, sin, rstd = ctx.saved_tensors
        nq, nkv, use_norm = ctx.cfg
        T = qkv.shape[0]
        dev = qkv.device
        dqkv = torch.empty(T, (nq + 2 * nkv) * 128, dtype=torch.bfloat16, device=dev)
        nparts = 296
        part = torch.empty(nparts, 256, dtype=torch.float32, device=dev)
        dw = torch.zeros(256, dtype=torch.float32, device=dev)

        def z(t, shp):
            return t.contiguous() if t is not None else torch.zeros(shp, dtype=torch.bfloat16, device=dev)

        lib().qk_norm_rope_bwd(z(dq, (T, nq, 128)), z(dk, (T, nkv, 128)), z(dv, (T, nkv, 128)), qkv,
                               qw, kw, pos, cos, sin, rstd, dqkv, part, dw, nq, nkv, use_norm)
        dqw = dw[:128].to(qw.dtype) if (use_norm and qw is not None) else None
        dkw = dw[128:].to(kw.dtype) if (use_norm and kw is not None) else None
        return dqkv, dqw, dkw, None, None, None, None, None, None, None


def qk_norm_rope(qkv, qw, kw, pos, cos, sin, nq, nkv, eps=1e-6, use_norm=True):
    """qkv [T, (nq+2nkv)*128] -> q [T,nq,128], k [T,nkv,128], v [T,nkv,128] with per-head
    RMSNorm (Qwen3 QK-norm) and rotary embedding at positions `pos` (int32 [T])."""
    if not use_native(qkv):
        return qk_norm_rope_ref(qkv, qw, kw, pos, cos, sin, nq, nkv, eps, use_norm)
    return _QKNormRope.apply(qkv, qw, kw, pos, cos, sin, nq, nkv, eps, use_norm)


def qk_norm_rope_to_cache(qkv, qw, kw, pos, cos, sin, nq, nkv, k_cache, v_cache, slots,
                          eps=1e-6, use_norm=True):
    """Inference form: returns q and writes k, v into cache rows `slots` (int64 [T])."""
    T = qkv.shape[0]
    if not use_native(qkv):
        q, k, v = qk_norm_rope_ref(qkv, qw, kw, pos, cos, sin, nq, nkv, eps, use_norm)
        k_cache[slots] = k
        v_cache[slots] = v
        return q
    q = torch.empty(T, nq, 128, dtype=torch.bfloat16, device=qkv.device)
    lib().qk_norm_rope_fwd(qkv, qw, kw, pos, cos, sin, q, k_cache, v_cache, slots, nkv * 128, None,
                           nq, nkv, eps, use_norm)
    return q


# ------------------------------------------------------------------------------------------
# SwiGLU
# ------------------------------------------------------------------------------------------
def swiglu_ref(gu: torch.Tensor) -> torch.Tensor:
    I = gu.shape[-1] // 2
    g, u = gu[..., :I].float(), gu[..., I:].float()
    return (torch.nn.functional.silu(g).to(gu.dtype).float() * u).to(gu.dtype)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        out = torch.empty(*gu.shape[:-1], gu.shape[-1] // 2, dtype=gu.dtype, device=gu.device)
        lib().swiglu_fwd(gu, out, None)
        ctx.save_for_backward(gu)
        return out

    @staticmethod
    def backward(ctx, dout):
        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        lib().swiglu_bwd(gu, dout.contiguous(), dgu, None)
        return dgu


def swiglu_bwd_raw(gu: torch.Tensor, dout: torch.Tensor) -> torch.Tensor:
    """d(gu) of the SwiGLU given its output grad (no autograd)."""
    if not use_native(gu):
        g = gu.detach().requires_grad_(True)
        with torch.enable_grad():
            swiglu_ref(g).backward(dout)
        return g.grad
    dgu = torch.empty_like(gu)
    lib().swiglu_bwd(gu, dout, dgu, None)
    return dgu


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up over the two halves of the last dim ([gate | up])."""
    if not use_native(gu):
        return swiglu_ref(gu)
    return _SwiGLU.apply(gu)
