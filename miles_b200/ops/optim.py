"""Adam(W) update and deterministic gradient-norm reduction (csrc/rl_ops.cu).

The clip coefficient is computed on the device from the squared norm, so a whole optimizer step
(norm -> clip -> update) runs without a host synchronisation.
"""
from __future__ import annotations

import torch

from miles_b200.ops._lib import lib, use_native


def sqnorm_(x: torch.Tensor, out: torch.Tensor, part: torch.Tensor | None = None) -> None:
    """out[0] += ||x||^2 (fixed-order reduction)."""
    if not use_native(x):
        out += x.float().pow(2).sum()
        return
    if part is None:
        part = torch.empty(148 * 8, dtype=torch.float32, device=x.device)
    lib().sqnorm(x.reshape(-1), part, out)


def nonfinite_(x: torch.Tensor, flag: torch.Tensor) -> None:
    if not use_native(x):
        if not torch.isfinite(x).all():
            flag.fill_(1.0)
        return
    lib().nonfinite(x.reshape(-1), flag)


def adam_(param: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor, *,
          master: torch.Tensor | None, lr: float, betas=(0.9, 0.999), eps: float = 1e-8,
          weight_decay: float = 0.0, step: int = 1, sqnorm: torch.Tensor | None = None,
          max_norm: float = 0.0, inv_loss_scale: float = 1.0, seed: int = 0,
          skip: torch.Tensor | None = None) -> None:
    """In-place AdamW on flat buffers. param bf16; master fp32 or None (stochastic rounding)."""
    if not use_native(param):
        if skip is not None and float(skip) != 0:
            return
        g = grad.float() * inv_loss_scale
        if sqnorm is not None and max_norm > 0:
            nrm = float(sqnorm.sqrt()) * inv_loss_scale
            g = g * min(1.0, max_norm / (nrm + 1e-6))
        b1, b2 = betas
        mf = m.float().mul(b1).add(g, alpha=1 - b1)
        vf = v.float().mul(b2).addcmul(g, g, value=1 - b2)
        upd = (mf / (1 - b1 ** step)) / ((vf / (1 - b2 ** step)).sqrt() + eps)
        w0 = master if master is not None else param.float()
        w1 = w0 - lr * (upd + weight_decay * w0)
        if master is not None:
            master.copy_(w1)
        param.copy_(w1.to(param.dtype))
        m.copy_(mf.to(m.dtype))
        v.copy_(vf.to(v.dtype))
        return
    lib().adam(param, master, m, v, grad, lr, betas[0], betas[1], eps, weight_decay, step, sqnorm,
               max_norm, inv_loss_scale, seed, skip)
