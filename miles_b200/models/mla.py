"""Multi-head latent attention (DeepSeek-V2/V3 style) for the transformer.

Per token: q = x Wq (or the low-rank Wq_b rmsnorm(x Wq_a)), split into a no-position part
(qk_nope_head_dim) and a rotary part (qk_rope_head_dim) per head; the keys and values come
from a shared latent c = rmsnorm((x Wkv_a)[:kv_lora_rank]) plus one rotary key k_pe shared by all
heads: [k_nope | v] = c Wkv_b per head, k = [k_nope | k_pe].

  * training / prefill materialise k and v and run causal attention per sequence
    (head dims qk = nope + rope, v = v_head_dim, which the head-dim-128 tcgen05 kernels do not
    cover: this path uses PyTorch's scaled_dot_product_attention);
  * the KV cache stores only [c | k_pe] (kv_lora_rank + qk_rope_head_dim values per token, one
    "head"), and decode runs the absorbed form (on GPUs in csrc/mla_decode.cu, straight from the
    paged cache): q_nope is mapped into latent space by the key
    half of Wkv_b, scores are q_lat . c + q_pe . k_pe, the value is read in latent space and
    mapped out by the value half of Wkv_b. Decode therefore never expands the cache.

Decode and training compute the same function through different operation orders, so MLA
rollout log-probs are not bitwise equal to the trainer's (the importance-sampling corrections
apply); the Qwen3 family keeps its bitwise parity.

DSA (DeepSeek-V3.2 / GLM-5 sparse attention, when `index_topk` > 0): a lightning indexer scores
every (query, key) pair as sum_h w[t, h] * relu(q_I[t, h] . k_I[s]) (q_I from the query latent,
one LayerNorm'ed key k_I per token, per-head weights w from the hidden state), and each query
attends only to its `index_topk` best-scoring causal keys. Training / prefill mask the dense
attention to those keys; decode scores the cached indexer keys (stored next to the latent in the
cache row) and masks the absorbed scores the same way. The top-k selection is discrete, so the
indexer parameters get no gradient from the policy loss.

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

from miles_b200.parallel.tp import copy_to_tp, reduce_from_tp


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of the latent vectors (kv_lora_rank / q_lora_rank wide: sizes the fused norm
    kernel is not built for), fp32 arithmetic, result in x's dtype."""
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


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
    if cfg.index_topk:  # DSA lightning indexer (replicated under TP)
        if not cfg.q_lora_rank:
            raise ValueError("the DSA indexer reads the low-rank query latent (q_lora_rank > 0)")
        nI, dI = cfg.index_n_heads, cfg.index_head_dim
        out += [(p + "indexer.wq_b.weight", (nI * dI, cfg.q_lora_rank), "normal"),
                (p + "indexer.wk.weight", (dI, H), "normal"),
                (p + "indexer.k_norm.weight", (dI,), "ones"),
                (p + "indexer.k_norm.bias", (dI,), "zeros"),
                (p + "indexer.weights_proj.weight", (nI, H), "normal")]
    out += [(p + "kv_a_proj_with_mqa.weight", (r + dr, H), "normal"),
            (p + "kv_a_layernorm.weight", (r,), "ones"),
            (p + "kv_b_proj.weight", (nh * (dn + dv), r), "normal"),
            (p + "o_proj.weight", (H, nh * dv), "normal")]
    return out


def _rope(x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
          interleaved: bool = False) -> torch.Tensor:
    """Rotate-half RoPE over the last dim of x [T, ..., d] at positions pos [T]. `interleaved`:
    the rotary pairs are adjacent dims (x0, x1), (x2, x3), ... and are first gathered into the
    rotate-half layout (the result stays in that layout)."""
    if interleaved:
        shp = x.shape
        x = x.reshape(*shp[:-1], shp[-1] // 2, 2).transpose(-1, -2).reshape(shp)
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
    # ------------------------------------------------------------------ DSA indexer
    def _index_q(self, i: int, qa: torch.Tensor, pos: torch.Tensor):
        """Indexer queries [T, nI, dI] (rotary on the first qk_rope_head_dim dims)."""
        cfg = self.cfg
        p = f"layers.{i}.self_attn.indexer."
        q = F.linear(qa.float(), self.m.params[p + "wq_b.weight"].float())
        q = q.view(qa.shape[0], cfg.index_n_heads, cfg.index_head_dim)
        return self._index_rope(q, pos)

    def _index_k(self, i: int, x: torch.Tensor, pos: torch.Tensor):
        """Indexer keys [T, dI] (LayerNorm, rotary on the first qk_rope_head_dim dims)."""
        cfg, P = self.cfg, self.m.params
        p = f"layers.{i}.self_attn.indexer."
        k = F.linear(x.float(), P[p + "wk.weight"].float())
        k = F.layer_norm(k, (cfg.index_head_dim,), P[p + "k_norm.weight"].float(),
                         P[p + "k_norm.bias"].float(), 1e-6)
        return self._index_rope(k, pos)

    def _index_rope(self, t: torch.Tensor, pos: torch.Tensor):
        """Rotary (rotate-half) on the first qk_rope_head_dim dims of the indexer heads."""
        dr = self.cfg.qk_rope_head_dim
        return torch.cat([_rope(t[..., :dr], pos, self.cos, self.sin), t[..., dr:]], -1)

    def _index_weights(self, i: int, x: torch.Tensor):
        cfg = self.cfg
        w = F.linear(x.float(), self.m.params[f"layers.{i}.self_attn.indexer.weights_proj.weight"].float())
        return w * (cfg.index_n_heads ** -0.5) * (cfg.index_head_dim ** -0.5)

    @staticmethod
    def _index_scores(qI, wI, kI):
        """[Tq, Tk] indexer scores sum_h w[t, h] relu(q_I[t, h] . k_I[s]), in fp64 so that the
        training and decode forms (different contraction shapes) select the same keys except at
        exact ties."""
        qI, kI, wI = qI.double(), kI.double(), wI.double()
        return torch.einsum("th,ths->ts", wI, torch.relu(torch.einsum("thd,sd->ths", qI, kI)))

    def _topk_keep(self, scores: torch.Tensor, valid: torch.Tensor) -> torch.Tensor:
        """Boolean mask of the index_topk best valid keys per query row."""
        k = min(self.cfg.index_topk, scores.shape[-1])
        sc = scores.masked_fill(~valid, float("-inf"))
        # ties (e.g. keys whose relu terms are all zero) go to the earlier key, in every path
        top = torch.sort(sc, dim=-1, descending=True, stable=True).indices[..., :k]
        keep = torch.zeros_like(valid).scatter_(-1, top, True)
        return keep & valid

    def _dsa_bias(self, i, x, qa, positions, cache, page_table, ctx_lens):
        """[B, maxk] additive bias of the DSA key selection over the cached indexer keys."""
        cfg = self.cfg
        B, page = x.shape[0], 64
        maxk = page_table.shape[1] * page
        t = torch.arange(maxk, device=x.device)
        rows = page_table.long()[:, t // page] * page + (t % page)[None, :]
        off = cfg.kv_lora_rank + cfg.qk_rope_head_dim
        kI = cache.k[i][:, 0, off:].index_select(0, rows.reshape(-1)).view(B, maxk, -1).double()
        qI, wI = self._index_q(i, qa, positions).double(), self._index_weights(i, x).double()
        scI = torch.einsum("bh,bhs->bs", wI, torch.relu(torch.einsum("bhd,bsd->bhs", qI, kI)))
        keep = self._topk_keep(scI, t[None, :] < ctx_lens[:, None].long())
        return torch.zeros(B, maxk, dtype=torch.float32, device=x.device).masked_fill(~keep, float("-inf"))

    def _q(self, i: int, x: torch.Tensor, pos: torch.Tensor, want_qa: bool = False):
        cfg, m = self.cfg, self.m
        p = f"layers.{i}.self_attn."
        qa = None
        if cfg.q_lora_rank:
            qa = rms_norm(m._lin(x, p + "q_a_proj.weight"), m.params[p + "q_a_layernorm.weight"], cfg.rms_eps)
            q = m._lin(copy_to_tp(qa, m.tp), p + "q_b_proj.weight")
        else:
            q = m._lin(copy_to_tp(x, m.tp), p + "q_proj.weight")
        q = q.view(x.shape[0], self.nh, cfg.qk_nope_head_dim + cfg.qk_rope_head_dim)
        q_nope, q_pe = q.split([cfg.qk_nope_head_dim, cfg.qk_rope_head_dim], -1)
        if want_qa:
            return q_nope, _rope(q_pe, pos, self.cos, self.sin, self.cfg.rope_interleave), qa
        return q_nope, _rope(q_pe, pos, self.cos, self.sin, self.cfg.rope_interleave)

    def _latent(self, i: int, x: torch.Tensor, pos: torch.Tensor):
        cfg, m = self.cfg, self.m
        p = f"layers.{i}.self_attn."
        kva = m._lin(x, p + "kv_a_proj_with_mqa.weight")
        c, k_pe = kva.split([cfg.kv_lora_rank, cfg.qk_rope_head_dim], -1)
        c = rms_norm(c.contiguous(), m.params[p + "kv_a_layernorm.weight"], cfg.rms_eps)
        return c, _rope(k_pe, pos, self.cos, self.sin, self.cfg.rope_interleave)

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
        q_nope, q_pe, qa = self._q(i, x, pos, want_qa=True)
        c, k_pe = self._latent(i, x, pos)
        dsa = cfg.index_topk > 0
        if dsa:
            with torch.no_grad():
                qI, kI, wI = self._index_q(i, qa.detach(), pos), self._index_k(i, x.detach(), pos), \
                    self._index_weights(i, x.detach())
        if cache is not None:
            row = [c, k_pe] + ([kI.to(c.dtype)] if dsa else [])
            cache.k[i].index_copy_(0, slots, torch.cat(row, -1).unsqueeze(1).to(cache.k[i].dtype))
        k, v = self._expand(i, c, k_pe)
        q = torch.cat([q_nope, q_pe], -1)
        o = self._sdpa(q, k, v, meta.cu_list, (qI, kI, wI) if dsa else None)
        return self._out(i, o.reshape(x.shape[0], -1), pending)

    def _sdpa(self, q, k, v, cu, index=None):
        """Causal attention per sequence of the packed rows (q, k, v [T, heads, D]); with the
        DSA indexer inputs (qI, kI, wI over the same rows) only each query's top-k keys."""
        o = torch.empty(q.shape[0], q.shape[1], v.shape[-1], dtype=q.dtype, device=q.device)
        outs = []
        for b in range(len(cu) - 1):
            s, e = cu[b], cu[b + 1]
            if e == s:
                continue
            qs, ks, vs = (t[s:e].transpose(0, 1).unsqueeze(0) for t in (q, k, v))
            if index is not None:
                qI, kI, wI = index
                L = e - s
                causal = torch.ones(L, L, dtype=torch.bool, device=q.device).tril()
                keep = self._topk_keep(self._index_scores(qI[s:e], wI[s:e], kI[s:e]), causal)
                o_b = F.scaled_dot_product_attention(qs, ks, vs, attn_mask=keep, scale=self.scale)
            else:
                o_b = F.scaled_dot_product_attention(qs, ks, vs, is_causal=True, scale=self.scale)
            outs.append(o_b[0].transpose(0, 1))
        return torch.cat(outs, 0) if outs else o

    def attn_sp(self, i: int, x: torch.Tensor, meta) -> torch.Tensor:
        """Sequence-parallel training attention: x holds this TP rank's rows, the result is
        this rank's rows of the o_proj output (reduce-scattered). The replicated down
        projections run on the local rows and the low-rank latents (q_a output, compressed KV
        and the shared rotary key: q_lora_rank + kv_lora_rank + qk_rope_head_dim wide) are
        all-gathered instead of the hidden state; the up projections then run on all rows for
        this rank's heads. The gather's backward reduce-scatters the latent gradients."""
        from miles_b200.parallel.tp import sp_gather

        cfg, m, tp = self.cfg, self.m, self.m.tp
        p = f"layers.{i}.self_attn."
        pos = meta.positions
        R = x.shape[0]
        T = R * tp.size
        lo = tp.rank * R
        dn, dr = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim
        qa = None
        if cfg.q_lora_rank:
            qa = sp_gather(rms_norm(m._lin(x, p + "q_a_proj.weight"), m.params[p + "q_a_layernorm.weight"],
                                    cfg.rms_eps), tp)
            q = m._lin(qa, p + "q_b_proj.weight")
        else:
            q = m._lin(sp_gather(x, tp), p + "q_proj.weight")
        q_nope, q_pe = q.view(T, self.nh, dn + dr).split([dn, dr], -1)
        q = torch.cat([q_nope, _rope(q_pe, pos, self.cos, self.sin, cfg.rope_interleave)], -1)
        kva = m._lin(x, p + "kv_a_proj_with_mqa.weight")
        c, k_pe = kva.split([cfg.kv_lora_rank, dr], -1)
        c = rms_norm(c.contiguous(), m.params[p + "kv_a_layernorm.weight"], cfg.rms_eps)
        lat = sp_gather(torch.cat([c, k_pe], -1), tp)
        c, k_pe = lat.split([cfg.kv_lora_rank, dr], -1)
        k_pe = _rope(k_pe, pos, self.cos, self.sin, cfg.rope_interleave)
        kv = m._lin(c.contiguous(), p + "kv_b_proj.weight").view(T, self.nh, dn + cfg.v_head_dim)
        k_nope, v = kv.split([dn, cfg.v_head_dim], -1)
        k = torch.cat([k_nope, k_pe[:, None, :].expand(-1, self.nh, -1)], -1)
        index = None
        if cfg.index_topk > 0:
            with torch.no_grad():
                pl = pos[lo:lo + R]
                index = (self._index_q(i, qa.detach(), pos),
                         sp_gather(self._index_k(i, x.detach(), pl), tp),
                         sp_gather(self._index_weights(i, x.detach()), tp))
        o = self._sdpa(q, k, v.contiguous(), meta.cu_list, index)
        return m._row_rs(o.reshape(T, -1), p + "o_proj.weight")

    def attn_cp(self, i: int, x: torch.Tensor, meta, pos: torch.Tensor, cp) -> torch.Tensor:
        """Context-parallel training attention: x holds this CP rank's rows of the padded batch.
        The per-head q / k / v (after the latent up-projection) go through the head all-to-all
        (all rows, 1 / CP of the heads per rank); the DSA indexer's inputs, computed without
        gradient, are all-gathered so that every rank selects the same top-k keys over the
        whole sequence (the reference's allgather-CP keeps the indexer global the same way)."""
        from miles_b200.parallel.cp import all_gather_rows, heads_to_tokens, tokens_to_heads

        cfg = self.cfg
        q_nope, q_pe, qa = self._q(i, x, pos, want_qa=True)
        c, k_pe = self._latent(i, x, pos)
        index = None
        if cfg.index_topk > 0:
            with torch.no_grad():
                index = tuple(all_gather_rows(t, cp) for t in (
                    self._index_q(i, qa.detach(), pos), self._index_k(i, x.detach(), pos),
                    self._index_weights(i, x.detach())))
        k, v = self._expand(i, c, k_pe)
        q = torch.cat([q_nope, q_pe], -1)
        oh = self._sdpa(tokens_to_heads(q, cp), tokens_to_heads(k, cp), tokens_to_heads(v, cp),
                        meta.cu_list, index)
        return self._out(i, heads_to_tokens(oh, cp).reshape(x.shape[0], -1), False)

    # ------------------------------------------------------------------ decode (absorbed)
    def decode(self, i: int, x: torch.Tensor, positions: torch.Tensor, cache, page_table: torch.Tensor,
               ctx_lens: torch.Tensor, slots: torch.Tensor, pending: bool = False):
        cfg = self.cfg
        B = x.shape[0]
        nh, dn, dv, r = self.nh, cfg.qk_nope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
        q_nope, q_pe, qa = self._q(i, x, positions, want_qa=True)
        c, k_pe = self._latent(i, x, positions)
        dsa = cfg.index_topk > 0
        row = [c, k_pe]
        if dsa:
            row.append(self._index_k(i, x, positions).to(c.dtype))
        cache.k[i].index_copy_(0, slots, torch.cat(row, -1).unsqueeze(1).to(cache.k[i].dtype))
        w = self.m.params[f"layers.{i}.self_attn.kv_b_proj.weight"].view(nh, dn + dv, r)
        w_uk, w_uv = w[:, :dn, :], w[:, dn:, :]
        q_lat = torch.einsum("bhn,hnc->bhc", q_nope.float(), w_uk.float())
        from miles_b200.ops._lib import lib, use_native

        if use_native(x):
            # csrc/mla_decode.cu reads the paged latent cache directly; DSA passes its key
            # selection as an additive bias (0 kept, -inf dropped)
            bias = None
            if dsa:
                bias = self._dsa_bias(i, x, qa, positions, cache, page_table, ctx_lens)
            o_lat = torch.empty(B, nh, r, dtype=torch.float32, device=x.device)
            lib().mla_decode(q_lat.contiguous(), q_pe.float().contiguous(), cache.k[i][:, 0, :],
                             page_table.int().contiguous(), ctx_lens.int().contiguous(), bias,
                             self.scale, o_lat)
            o = torch.einsum("bhc,hvc->bhv", o_lat, w_uv.float()).to(x.dtype)
            return self._out(i, o.reshape(B, -1), pending)
        page = 64
        maxk = page_table.shape[1] * page
        t = torch.arange(maxk, device=x.device)
        rows = page_table.long()[:, t // page] * page + (t % page)[None, :]  # [B, maxk] cache rows
        width = cache.k[i].shape[-1]
        lat = cache.k[i][:, 0, :].index_select(0, rows.reshape(-1)).view(B, maxk, width)
        ck, kp = lat[..., :r].float(), lat[..., r:r + cfg.qk_rope_head_dim].float()
        sc = (torch.einsum("bhc,btc->bht", q_lat, ck) + torch.einsum("bhd,btd->bht", q_pe.float(), kp)) * self.scale
        valid = t[None, :] < ctx_lens[:, None].long()  # [B, maxk]
        if dsa:
            kI = lat[..., r + cfg.qk_rope_head_dim:].float()                       # [B, maxk, dI]
            qI, wI = self._index_q(i, qa, positions), self._index_weights(i, x)   # [B, nI, dI], [B, nI]
            qI, kI, wI = qI.double(), kI.double(), wI.double()
            scI = torch.einsum("bh,bhs->bs", wI, torch.relu(torch.einsum("bhd,bsd->bhs", qI, kI)))
            valid = self._topk_keep(scI, valid)
        sc = sc.masked_fill(~valid[:, None, :], float("-inf"))
        pr = torch.softmax(sc, -1)
        o_lat = torch.einsum("bht,btc->bhc", pr, ck)
        o = torch.einsum("bhc,hvc->bhv", o_lat, w_uv.float()).to(x.dtype)
        return self._out(i, o.reshape(B, -1), pending)
