"""Multi-head latent attention (DeepSeek-V2/V3 style) for the transformer.

Per token: q = x Wq (or the low-rank Wq_b rmsnorm(x Wq_a)), split into a no-position part
(qk_nope_head_dim) and a rotary part (qk_rope_head_dim) per head; the keys and values come
from a shared latent c = rmsnorm((x Wkv_a)[:kv_lora_rank]) plus one rotary key k_pe shared by all
heads: [k_nope | v] = c Wkv_b per head, k = [k_nope | k_pe].

  * training / prefill materialise k and v and run causal attention per sequence
    (head dims qk = nope + rope, v = v_head_dim, which the head-dim-128 tcgen05 kernels do not
    cover: this path uses PyTorch's scaled_dot_product_attention);
  * the KV cache stores only [c | k_pe] (kv_lora_rank + qk_rope_head_dim values per token, one
    "head"), and decode runs the absorbed form: q_nope is mapped into latent space by the key
    half of Wkv_b, scores are q_lat . c + q_pe . k_pe, the value is read in latent space and
    mapped out by the value half of Wkv_b. Decode therefore never expands the cache.

Decode and training compute the same function through different operation orders, so MLA
rollout log-probs are not bitwise equal to the trainer's (the importance-sampling corrections
apply); the Qwen3 family keeps its bitwise parity.

Parameter names follow the HF DeepSeek-V3 layout (q_proj or q_a_proj / q_a_layernorm / q_b_proj,
kv_a_proj_with_mqa, kv_a_layernorm, kv_b_proj, o_proj).

Reference: the DeepSeek-V3 / GLM MLA model support of the reference goes through Megatron's
MLA layer and SGLang's MLA backends (miles_plugins/models/glm5/glm5.py, mbridge deepseek_v32,
megatron_to_hf/deepseekv3.py).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from miles_b200.ops.norm import rms_norm
from miles_b200.parallel.tp import copy_to_tp, reduce_from_tp


def mla_param_shapes(cfg, p: str, tp_size: int = 1):
    """Parameter shapes of one MLA layer; tensor parallelism splits the heads (q_proj /
    q_b_proj / kv_b_proj rows, o_proj columns) and replicates the latent projections."""
    H, nh = cfg.hidden_size, cfg.num_heads // tp_size
    dn, dr, dv, r = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
    out = []
    if cfg.q_lora_rank:
        out += [(p + "q_a_proj.weight", (cfg.q_lora_rank, H), "normal"),
                (p + "q_a_layernorm.weight", (cfg.q_lora_rank,), "ones"),
                (p + "q_b_proj.weight", (nh * (dn + dr), cfg.q_lora_rank), "normal")]
    else:
        out.append((p + "q_proj.weight", (nh * (dn + dr), H), "normal"))
    out += [(p + "kv_a_proj_with_mqa.weight", (r + dr, H), "normal"),
            (p + "kv_a_layernorm.weight", (r,), "ones"),
            (p + "kv_b_proj.weight", (nh * (dn + dv), r), "normal"),
            (p + "o_proj.weight", (H, nh * dv), "normal")]
    return out


def _rope(x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE over the last dim of x [T, ..., d] at positions pos [T]."""
    d = x.shape[-1] // 2
    c = cos.index_select(0, pos.long())
    s = sin.index_select(0, pos.long())
    while c.dim() < x.dim():
        c, s = c.unsqueeze(1), s.unsqueeze(1)
    x1, x2 = x[..., :d].float(), x[..., d:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)


class MLA:
    def __init__(self, model):
        cfg = model.cfg
        self.m = model
        self.cfg = cfg
        self.nh = cfg.num_heads // model.tp_size  # this rank's heads
        from miles_b200.ops.norm import rope_tables

        self.cos, self.sin = rope_tables(cfg.max_position, cfg.qk_rope_head_dim, cfg.rope_theta,
                                         model.device, cfg.rope_scaling)
        mscale = 1.0
        if cfg.rope_scaling and cfg.rope_scaling.get("mscale_all_dim"):
            f = float(cfg.rope_scaling.get("factor", 1.0))
            mscale = 0.1 * float(cfg.rope_scaling["mscale_all_dim"]) * math.log(f) + 1.0 if f > 1 else 1.0
        self.scale = mscale * mscale / math.sqrt(cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)

    # ------------------------------------------------------------------ projections
    def _q(self, i: int, x: torch.Tensor, pos: torch.Tensor):
        cfg, m = self.cfg, self.m
        p = f"layers.{i}.self_attn."
        if cfg.q_lora_rank:
            qa = rms_norm(m._lin(x, p + "q_a_proj.weight"), m.params[p + "q_a_layernorm.weight"], cfg.rms_eps)
            q = m._lin(copy_to_tp(qa, m.tp), p + "q_b_proj.weight")
        else:
            q = m._lin(copy_to_tp(x, m.tp), p + "q_proj.weight")
        q = q.view(x.shape[0], self.nh, cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
        q_nope, q_pe = q.split([cfg.qk_nope_head_dim, cfg.qk_rope_head_dim], -1)
        return q_nope, _rope(q_pe, pos, self.cos, self.sin)

    def _latent(self, i: int, x: torch.Tensor, pos: torch.Tensor):
        cfg, m = self.cfg, self.m
        p = f"layers.{i}.self_attn."
        kva = m._lin(x, p + "kv_a_proj_with_mqa.weight")
        c, k_pe = kva.split([cfg.kv_lora_rank, cfg.qk_rope_head_dim], -1)
        c = rms_norm(c.contiguous(), m.params[p + "kv_a_layernorm.weight"], cfg.rms_eps)
        return c, _rope(k_pe, pos, self.cos, self.sin)

    def _expand(self, i: int, c: torch.Tensor, k_pe: torch.Tensor):
        cfg, m = self.cfg, self.m
        kv = m._lin(copy_to_tp(c, m.tp), f"layers.{i}.self_attn.kv_b_proj.weight").view(
            c.shape[0], self.nh, cfg.qk_nope_head_dim + cfg.v_head_dim)
        k_nope, v = kv.split([cfg.qk_nope_head_dim, cfg.v_head_dim], -1)
        k = torch.cat([k_nope, copy_to_tp(k_pe, m.tp)[:, None, :].expand(-1, self.nh, -1)], -1)
        return k, v

    # ------------------------------------------------------------------ training / prefill
    def _out(self, i: int, o: torch.Tensor, pending: bool):
        """o_proj (row parallel): the reduced output, or (pending) what the caller reduces."""
        name = f"layers.{i}.self_attn.o_proj.weight"
        if pending:
            return self.m._pending_out(o, name)
        return reduce_from_tp(self.m._lin(o, name), self.m.tp)

    def attn(self, i: int, x: torch.Tensor, meta, cache=None, slots=None, pending: bool = False):
        cfg = self.cfg
        pos = meta.positions
        q_nope, q_pe = self._q(i, x, pos)
        c, k_pe = self._latent(i, x, pos)
        if cache is not None:
            cache.k[i].index_copy_(0, slots, torch.cat([c, k_pe], -1).unsqueeze(1).to(cache.k[i].dtype))
        k, v = self._expand(i, c, k_pe)
        q = torch.cat([q_nope, q_pe], -1)
        o = torch.empty(x.shape[0], self.nh, cfg.v_head_dim, dtype=x.dtype, device=x.device)
        outs = []
        cu = meta.cu_list
        for b in range(len(cu) - 1):
            s, e = cu[b], cu[b + 1]
            if e == s:
                continue
            qs, ks, vs = (t[s:e].transpose(0, 1).unsqueeze(0) for t in (q, k, v))
            outs.append(F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=self.scale)
                        [0].transpose(0, 1))
        o = torch.cat(outs, 0) if outs else o
        return self._out(i, o.reshape(x.shape[0], -1), pending)

    # ------------------------------------------------------------------ decode (absorbed)
    def decode(self, i: int, x: torch.Tensor, positions: torch.Tensor, cache, page_table: torch.Tensor,
               ctx_lens: torch.Tensor, slots: torch.Tensor, pending: bool = False):
        cfg = self.cfg
        B = x.shape[0]
        nh, dn, dv, r = self.nh, cfg.qk_nope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
        q_nope, q_pe = self._q(i, x, positions)
        c, k_pe = self._latent(i, x, positions)
        cache.k[i].index_copy_(0, slots, torch.cat([c, k_pe], -1).unsqueeze(1).to(cache.k[i].dtype))
        w = self.m.params[f"layers.{i}.self_attn.kv_b_proj.weight"].view(nh, dn + dv, r)
        w_uk, w_uv = w[:, :dn, :], w[:, dn:, :]
        q_lat = torch.einsum("bhn,hnc->bhc", q_nope.float(), w_uk.float())
        page = 64
        maxk = page_table.shape[1] * page
        t = torch.arange(maxk, device=x.device)
        rows = page_table.long()[:, t // page] * page + (t % page)[None, :]  # [B, maxk] cache rows
        lat = cache.k[i][:, 0, :].index_select(0, rows.reshape(-1)).view(B, maxk, r + cfg.qk_rope_head_dim)
        ck, kp = lat[..., :r].float(), lat[..., r:].float()
        sc = (torch.einsum("bhc,btc->bht", q_lat, ck) + torch.einsum("bhd,btd->bht", q_pe.float(), kp)) * self.scale
        sc = sc.masked_fill((t[None, :] >= ctx_lens[:, None].long())[:, None, :], float("-inf"))
        pr = torch.softmax(sc, -1)
        o_lat = torch.einsum("bht,btc->bhc", pr, ck)
        o = torch.einsum("bhc,hvc->bhv", o_lat, w_uv.float()).to(x.dtype)
        return self._out(i, o.reshape(B, -1), pending)
