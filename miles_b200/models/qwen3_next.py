"""Softmax attention with separate q / k / v projections, for the families whose attention the
fused qkv + QK-norm/RoPE kernel path does not cover: Qwen3-Next's gated attention and GLM-4.5's
attention with projection biases and half-width rotary.

Every `linear_attn_interval`-th layer of a Qwen3-Next model keeps softmax attention with three
differences from Qwen3's:
  * q_proj also produces a per-head output gate: q_proj(x) viewed [T, nq, 2 D] = [q | gate];
    the attention output is multiplied by sigmoid(gate) before o_proj;
  * rotary embedding on the first D * partial_rotary_factor dims of each head only;
  * the model's RMSNorms are zero-centred in the checkpoint (y = x_hat * (1 + w)); the HF
    loader stores 1 + w, so the ordinary norm kernels apply unchanged.
q / k / v are separate projections (HF names); QK-norm per head. Under TP each rank holds
1 / TP of the query and KV heads (column-parallel q / k / v with their biases, row-parallel
o_proj). Attention uses the tcgen05
varlen / paged-decode kernels when the head size is 128 and the device is a GPU, PyTorch
otherwise (Qwen3-Next's 256-wide heads).

Reference: the Qwen3-Next model support of the reference (miles_plugins/models/qwen3_next.py,
HF-style attention through Megatron / SGLang); HF transformers' Qwen3NextAttention semantics.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from miles_b200.models.mla import _rope


def gated_attn_param_shapes(cfg, p: str, tp: int = 1):
    """Shapes of this TP rank's slice: q / k / v / o projections hold 1 / tp of the heads."""
    H, D, nq, nkv = cfg.hidden_size, cfg.head_dim, cfg.num_heads // tp, cfg.num_kv_heads // tp
    g = 2 if cfg.attn_output_gate else 1
    out = [(p + "q_proj.weight", (g * nq * D, H), "normal"),
           (p + "k_proj.weight", (nkv * D, H), "normal"),
           (p + "v_proj.weight", (nkv * D, H), "normal"),
           (p + "o_proj.weight", (H, nq * D), "normal")]
    if cfg.attention_bias:
        out += [(p + "q_proj.bias", (g * nq * D,), "zeros"), (p + "k_proj.bias", (nkv * D,), "zeros"),
                (p + "v_proj.bias", (nkv * D,), "zeros")]
    return out


def _head_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class GatedAttention:
    def __init__(self, model):
        from miles_b200.ops.norm import rope_tables

        self.m = model
        self.cfg = cfg = model.cfg
        self.D = cfg.head_dim
        self.rot = int(cfg.head_dim * cfg.partial_rotary_factor)
        self.cos, self.sin = rope_tables(cfg.max_position, self.rot, cfg.rope_theta, model.device,
                                         cfg.rope_scaling)

    def _native(self, x) -> bool:
        from miles_b200.ops._lib import use_native

        return self.D == 128 and use_native(x)

    def _qkv(self, i: int, x: torch.Tensor, pos: torch.Tensor, tp_copy: bool = True):
        from miles_b200.parallel.tp import copy_to_tp

        cfg, m, D = self.cfg, self.m, self.D
        nq, nkv = m.nq, m.nkv  # this TP rank's heads
        p = f"layers.{i}.self_attn."
        T = x.shape[0]
        xt = copy_to_tp(x, m.tp) if tp_copy else x

        def proj(name):
            y = m._lin(xt, p + name + ".weight")
            b = m.params.get(p + name + ".bias")
            return y if b is None else y + b.to(y.dtype)

        if cfg.attn_output_gate:
            qg = proj("q_proj").view(T, nq, 2 * D)
            q, gate = qg[..., :D], qg[..., D:].reshape(T, nq * D)
        else:
            q, gate = proj("q_proj").view(T, nq, D), None
        k = proj("k_proj").view(T, nkv, D)
        v = proj("v_proj").view(T, nkv, D)
        if cfg.qk_norm:
            q = _head_norm(q, m.params[p + "q_norm.weight"], cfg.rms_eps)
            k = _head_norm(k, m.params[p + "k_norm.weight"], cfg.rms_eps)
        r = self.rot
        il = cfg.rope_interleave  # GLM-4: adjacent-pair rotary (same scores, permuted layout)
        q = torch.cat([_rope(q[..., :r], pos, self.cos, self.sin, il), q[..., r:]], -1).contiguous()
        k = torch.cat([_rope(k[..., :r], pos, self.cos, self.sin, il), k[..., r:]], -1).contiguous()
        return q, k, v.contiguous(), gate

    def _out(self, i: int, o: torch.Tensor, gate, pending: bool = False):
        """o_proj (row parallel under TP): the reduced output, or (pending) the partial /
        deferred product that the caller's residual add + norm reduces."""
        from miles_b200.parallel.tp import reduce_from_tp

        o = o.reshape(o.shape[0], -1)
        if gate is not None:
            o = o * torch.sigmoid(gate.float()).to(o.dtype)
        name = f"layers.{i}.self_attn.o_proj.weight"
        if pending:
            return self.m._pending_out(o, name)
        return reduce_from_tp(self.m._lin(o, name), self.m.tp)

    def _sdpa(self, q, k, v, cu):
        rep = q.shape[1] // k.shape[1]  # the heads passed in (a CP head slice may hold one KV head)
        outs = []
        for b in range(len(cu) - 1):
            s, e = cu[b], cu[b + 1]
            if e == s:
                continue
            qs = q[s:e].transpose(0, 1)[None]
            ks = k[s:e].repeat_interleave(rep, 1).transpose(0, 1)[None]
            vs = v[s:e].repeat_interleave(rep, 1).transpose(0, 1)[None]
            outs.append(F.scaled_dot_product_attention(qs, ks, vs, is_causal=True,
                                                       scale=1.0 / math.sqrt(self.D))[0].transpose(0, 1))
        return torch.cat(outs, 0)

    def attn(self, i: int, x: torch.Tensor, meta, cache=None, slots=None,
             pending: bool = False) -> torch.Tensor:
        q, k, v, gate = self._qkv(i, x, meta.positions)
        if cache is not None:
            cache.k[i].index_copy_(0, slots, k.to(cache.k[i].dtype))
            cache.v[i].index_copy_(0, slots, v.to(cache.v[i].dtype))
        if self._native(x):
            from miles_b200.ops.attention import varlen_attention

            o = varlen_attention(q, k, v, meta)
        else:
            o = self._sdpa(q, k, v, meta.cu_list)
        return self._out(i, o, gate, pending)

    def attn_sp(self, i: int, x: torch.Tensor, meta) -> torch.Tensor:
        """Sequence parallel: x holds this TP rank's rows; projections on the all-gathered rows
        (the gather's backward reduce-scatters), o_proj ends in a reduce-scatter."""
        from miles_b200.parallel.tp import sp_gather

        xf = sp_gather(x, self.m.tp)
        q, k, v, gate = self._qkv(i, xf, meta.positions, tp_copy=False)
        if self._native(x):
            from miles_b200.ops.attention import varlen_attention

            o = varlen_attention(q, k, v, meta)
        else:
            o = self._sdpa(q, k, v, meta.cu_list)
        o = o.reshape(xf.shape[0], -1)
        if gate is not None:
            o = o * torch.sigmoid(gate.float()).to(o.dtype)
        return self.m._row_rs(o, f"layers.{i}.self_attn.o_proj.weight")

    def decode(self, i: int, x: torch.Tensor, positions, cache, page_table, ctx_lens, slots,
               pending: bool = False):
        cfg = self.cfg
        q, k, v, gate = self._qkv(i, x, positions)
        cache.k[i].index_copy_(0, slots, k.to(cache.k[i].dtype))
        cache.v[i].index_copy_(0, slots, v.to(cache.v[i].dtype))
        if self._native(x):
            from miles_b200.ops.attention import decode_attention

            o = decode_attention(q, cache.k[i], cache.v[i], page_table, ctx_lens)
        else:
            page = 64
            B = x.shape[0]
            maxk = page_table.shape[1] * page
            t = torch.arange(maxk, device=x.device)
            rows = (page_table.long()[:, t // page] * page + (t % page)[None, :]).reshape(-1)
            nkv = self.m.nkv
            kc = cache.k[i].index_select(0, rows).view(B, maxk, nkv, self.D).float()
            vc = cache.v[i].index_select(0, rows).view(B, maxk, nkv, self.D).float()
            rep = self.m.nq // nkv
            kc, vc = kc.repeat_interleave(rep, 2), vc.repeat_interleave(rep, 2)
            sc = torch.einsum("bhd,bthd->bht", q.float(), kc) / math.sqrt(self.D)
            sc = sc.masked_fill((t[None, :] >= ctx_lens[:, None].long())[:, None, :], float("-inf"))
            o = torch.einsum("bht,bthd->bhd", torch.softmax(sc, -1), vc).to(x.dtype)
        return self._out(i, o, gate, pending)
