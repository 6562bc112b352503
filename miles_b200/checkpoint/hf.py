"""HuggingFace safetensors import / export with per-family name mapping.

Our flat parameter layout fuses projections (qkv_proj = [q; k; v], gate_up_proj = [gate; up],
experts.w1 = E x [gate; up], experts.w2 = E x down). The converters split / join them to the HF
names of Qwen2/Qwen3 (dense), Qwen3-MoE and DeepSeek-V3-style MoE checkpoints, stream shards of
at most `max_shard_bytes`, and write `model.safetensors.index.json`.

Reference: megatron_to_hf/* (qwen3moe.py:65-76 QKV split, gate/up chunk, expert indices,
router and e_score_correction_bias names), tools/convert_torch_dist_to_hf.py,
megatron_utils/model.py save_hf (:718-772).
"""
from __future__ import annotations

import json
import os
import warnings
from typing import Iterator

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from miles_b200.models.config import ModelConfig
from miles_b200.models.transformer import Transformer
from miles_b200.parallel.tp import model_tp, tp_gather_for, tp_slice_for


def to_hf_tensors(model: Transformer) -> Iterator[tuple[str, torch.Tensor]]:
    """Yield (hf_name, tensor) for every parameter, splitting fused projections. Under tensor
    parallelism the tensors are this rank's slices (miles_b200/parallel/tp.py: hf_shard_dim)."""
    cfg = model.cfg
    H, D, nq, nkv = cfg.hidden_size, cfg.head_dim, model.nq, model.nkv
    P = model.params
    pre = "model."
    if "embed_tokens.weight" in P:
        yield pre + "embed_tokens.weight", P["embed_tokens.weight"].data
    for i in list(model.layer_ids) + list(getattr(model, "mtp_ids", [])):
        L = f"layers.{i}."
        yield pre + L + "input_layernorm.weight", P[L + "input_layernorm.weight"].data
        yield pre + L + "post_attention_layernorm.weight", P[L + "post_attention_layernorm.weight"].data
        if cfg.sandwich_norm:
            yield pre + L + "post_self_attn_layernorm.weight", P[L + "post_self_attn_layernorm.weight"].data
            yield pre + L + "post_mlp_layernorm.weight", P[L + "post_mlp_layernorm.weight"].data
        if cfg.layer_is_linear(i):  # Gated DeltaNet parameters carry their HF names
            for n in P:
                if not n.startswith(L + "linear_attn."):
                    continue
                if cfg.arch == "qwen3_5" and n.endswith(("in_proj_qkvz.weight", "in_proj_ba.weight")):
                    # Qwen3.5 stores the projections separately: [q; k; v], z, b, a
                    w = P[n].data
                    if n.endswith("qkvz.weight"):
                        vd = model.gdn.nv * cfg.linear_value_head_dim  # this TP rank's heads
                        yield pre + L + "linear_attn.in_proj_qkv.weight", w[: w.shape[0] - vd]
                        yield pre + L + "linear_attn.in_proj_z.weight", w[w.shape[0] - vd:]
                    else:
                        nv = model.gdn.nv
                        yield pre + L + "linear_attn.in_proj_b.weight", w[:nv]
                        yield pre + L + "linear_attn.in_proj_a.weight", w[nv:]
                    continue
                yield pre + n, P[n].data
        elif cfg.kv_lora_rank or cfg.uses_torch_attention:  # MLA / separate q,k,v: HF names already
            for n in P:
                if n.startswith(L + "self_attn."):
                    yield pre + n, P[n].data
        else:
            qkv = P[L + "self_attn.qkv_proj.weight"].data
            q, k, v = torch.split(qkv, [nq * D, nkv * D, nkv * D], 0)
            yield pre + L + "self_attn.q_proj.weight", q
            yield pre + L + "self_attn.k_proj.weight", k
            yield pre + L + "self_attn.v_proj.weight", v
            yield pre + L + "self_attn.o_proj.weight", P[L + "self_attn.o_proj.weight"].data
        if cfg.qk_norm and not cfg.kv_lora_rank and not cfg.layer_is_linear(i) and not cfg.uses_torch_attention:
            yield pre + L + "self_attn.q_norm.weight", P[L + "self_attn.q_norm.weight"].data
            yield pre + L + "self_attn.k_norm.weight", P[L + "self_attn.k_norm.weight"].data
        if cfg.layer_is_moe(i):
            yield pre + L + "mlp.gate.weight", P[L + "mlp.gate.weight"].data
            if L + "mlp.gate.e_score_correction_bias" in P:
                yield pre + L + "mlp.gate.e_score_correction_bias", P[L + "mlp.gate.e_score_correction_bias"].data
            w1 = P[L + "mlp.experts.w1"].data
            w2 = P[L + "mlp.experts.w2"].data
            I = w1.shape[1] // 2
            e0 = model.ep.first if getattr(model, "ep", None) is not None else 0  # global expert ids
            for e in range(w1.shape[0]):
                yield pre + L + f"mlp.experts.{e0 + e}.gate_proj.weight", w1[e, :I]
                yield pre + L + f"mlp.experts.{e0 + e}.up_proj.weight", w1[e, I:]
                yield pre + L + f"mlp.experts.{e0 + e}.down_proj.weight", w2[e]
            if cfg.shared_expert_intermediate_size:
                gu = P[L + "mlp.shared_expert.gate_up_proj.weight"].data
                Is = gu.shape[0] // 2
                yield pre + L + "mlp.shared_expert.gate_proj.weight", gu[:Is]
                yield pre + L + "mlp.shared_expert.up_proj.weight", gu[Is:]
                yield pre + L + "mlp.shared_expert.down_proj.weight", P[L + "mlp.shared_expert.down_proj.weight"].data
                yield pre + L + "mlp.shared_expert_gate.weight", P[L + "mlp.shared_expert_gate.weight"].data
            if cfg.num_shared_experts:
                gu = P[L + "mlp.shared_experts.gate_up_proj.weight"].data
                Is = gu.shape[0] // 2
                yield pre + L + "mlp.shared_experts.gate_proj.weight", gu[:Is]
                yield pre + L + "mlp.shared_experts.up_proj.weight", gu[Is:]
                yield pre + L + "mlp.shared_experts.down_proj.weight", P[L + "mlp.shared_experts.down_proj.weight"].data
        elif cfg.arch == "glm4":  # fused [gate; up] under its HF name
            yield pre + L + "mlp.gate_up_proj.weight", P[L + "mlp.gate_up_proj.weight"].data
            yield pre + L + "mlp.down_proj.weight", P[L + "mlp.down_proj.weight"].data
        else:
            gu = P[L + "mlp.gate_up_proj.weight"].data
            I = gu.shape[0] // 2
            yield pre + L + "mlp.gate_proj.weight", gu[:I]
            yield pre + L + "mlp.up_proj.weight", gu[I:]
            yield pre + L + "mlp.down_proj.weight", P[L + "mlp.down_proj.weight"].data
    for j in getattr(model, "mtp_ids", []):  # multi-token prediction extras (DeepSeek-V3 names)
        for n in ("enorm.weight", "hnorm.weight", "eh_proj.weight", "shared_head.norm.weight"):
            yield pre + f"layers.{j}." + n, P[f"layers.{j}." + n].data
    if "norm.weight" in P:
        yield pre + "norm.weight", P["norm.weight"].data
    if not cfg.tie_embeddings and "lm_head.weight" in P:
        yield "lm_head.weight", P["lm_head.weight"].data


_OFFSET_NORMS = ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_norm.weight",
                 "self_attn.k_norm.weight")


def _gdn_group_split(cfg):
    nk, nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
    r = nv // nk
    return nk, [cfg.linear_key_head_dim, cfg.linear_key_head_dim, r * cfg.linear_value_head_dim,
                r * cfg.linear_value_head_dim], [r, r]


def from_hf_layout(cfg: ModelConfig, name: str, t: torch.Tensor) -> torch.Tensor:
    """HF checkpoint tensor -> this framework's layout (identity for most tensors):
    zero-centred norms store 1 + w; Gated DeltaNet's in_proj_qkvz / in_proj_ba are regrouped
    from per-key-head-group interleaving into contiguous [q; k; v; z] / [b; a] blocks, and
    conv1d.weight drops its middle dim."""
    if cfg.norm_offset and (name.endswith(_OFFSET_NORMS) or name == "model.norm.weight"):
        return t.float() + 1.0
    if name.endswith("linear_attn.in_proj_qkvz.weight") or name.endswith("linear_attn.in_proj_ba.weight"):
        nk, sq, sb = _gdn_group_split(cfg)
        sizes = sq if name.endswith("qkvz.weight") else sb
        parts = t.view(nk, sum(sizes), -1).split(sizes, 1)
        return torch.cat([p.reshape(-1, t.shape[-1]) for p in parts], 0)
    if name.endswith("linear_attn.conv1d.weight") and t.dim() == 3:
        return t[:, 0, :]
    return t


def to_hf_layout(cfg: ModelConfig, name: str, t: torch.Tensor) -> torch.Tensor:
    """Inverse of from_hf_layout."""
    if cfg.norm_offset and (name.endswith(_OFFSET_NORMS) or name == "model.norm.weight"):
        return (t.float() - 1.0).to(t.dtype)
    if name.endswith("linear_attn.in_proj_qkvz.weight") or name.endswith("linear_attn.in_proj_ba.weight"):
        nk, sq, sb = _gdn_group_split(cfg)
        sizes = sq if name.endswith("qkvz.weight") else sb
        blocks = t.split([s * nk for s in sizes], 0)
        per = [b.view(nk, s, -1) for b, s in zip(blocks, sizes)]
        return torch.cat(per, 1).reshape(t.shape)
    if name.endswith("linear_attn.conv1d.weight") and t.dim() == 2:
        return t[:, None, :]
    return t


def hf_config_dict(cfg: ModelConfig) -> dict:
    d = {"vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size,
         "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
         "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
         "intermediate_size": cfg.intermediate_size, "rms_norm_eps": cfg.rms_eps,
         "rope_theta": cfg.rope_theta, "rope_scaling": cfg.rope_scaling,
         "rope_parameters": dict({"rope_theta": cfg.rope_theta, "rope_type": "default"},
                                 **(cfg.rope_scaling or {})),
         "max_position_embeddings": cfg.max_position, "tie_word_embeddings": cfg.tie_embeddings,
         "torch_dtype": "bfloat16"}
    d.update({k: None for k in ("pad_token_id", "bos_token_id", "eos_token_id")})
    d.update(cfg.extra.get("token_ids", {}))
    if cfg.arch == "qwen3_moe":
        d.update(model_type="qwen3_moe", architectures=["Qwen3MoeForCausalLM"],
                 num_experts=cfg.num_experts, num_local_experts=cfg.num_experts,
                 num_experts_per_tok=cfg.topk,
                 moe_intermediate_size=cfg.moe_intermediate_size, norm_topk_prob=cfg.norm_topk_prob,
                 decoder_sparse_step=1, mlp_only_layers=[])
    elif cfg.arch == "deepseek_v3":
        d.update(model_type="deepseek_v3", architectures=["DeepseekV3ForCausalLM"],
                 n_routed_experts=cfg.num_experts, num_experts_per_tok=cfg.topk,
                 moe_intermediate_size=cfg.moe_intermediate_size, n_shared_experts=cfg.num_shared_experts,
                 first_k_dense_replace=cfg.first_k_dense, scoring_func=cfg.router_score,
                 n_group=cfg.n_group, topk_group=cfg.topk_group,
                 routed_scaling_factor=cfg.routed_scaling_factor, norm_topk_prob=cfg.norm_topk_prob,
                 kv_lora_rank=cfg.kv_lora_rank, q_lora_rank=cfg.q_lora_rank or None,
                 qk_nope_head_dim=cfg.qk_nope_head_dim, qk_rope_head_dim=cfg.qk_rope_head_dim,
                 v_head_dim=cfg.v_head_dim, rope_interleave=cfg.rope_interleave)
        if cfg.index_topk:
            d.update(model_type="deepseek_v32", architectures=["DeepseekV32ForCausalLM"],
                     index_n_heads=cfg.index_n_heads, index_head_dim=cfg.index_head_dim,
                     index_topk=cfg.index_topk)
    elif cfg.arch == "glm4":
        d.update(model_type="glm4", architectures=["Glm4ForCausalLM"], attention_bias=cfg.attention_bias,
                 partial_rotary_factor=cfg.partial_rotary_factor)
        d["rope_parameters"]["partial_rotary_factor"] = cfg.partial_rotary_factor
    elif cfg.arch == "glm4_moe":
        d.update(model_type="glm4_moe", architectures=["Glm4MoeForCausalLM"],
                 n_routed_experts=cfg.num_experts, num_experts_per_tok=cfg.topk,
                 moe_intermediate_size=cfg.moe_intermediate_size, n_shared_experts=cfg.num_shared_experts,
                 first_k_dense_replace=cfg.first_k_dense, n_group=cfg.n_group, topk_group=cfg.topk_group,
                 routed_scaling_factor=cfg.routed_scaling_factor, norm_topk_prob=cfg.norm_topk_prob,
                 attention_bias=cfg.attention_bias, use_qk_norm=cfg.qk_norm,
                 partial_rotary_factor=cfg.partial_rotary_factor)
        d["rope_parameters"]["partial_rotary_factor"] = cfg.partial_rotary_factor
    elif cfg.arch in ("qwen3_next", "qwen3_5"):
        if cfg.arch == "qwen3_5":
            d.update(model_type="qwen3_5_moe_text" if cfg.is_moe else "qwen3_5_text",
                     architectures=["Qwen3_5MoeForCausalLM" if cfg.is_moe else "Qwen3_5ForCausalLM"])
        else:
            d.update(model_type="qwen3_next", architectures=["Qwen3NextForCausalLM"])
        d.update(
                 full_attention_interval=cfg.linear_attn_interval,
                 linear_num_key_heads=cfg.linear_num_key_heads,
                 linear_num_value_heads=cfg.linear_num_value_heads,
                 linear_key_head_dim=cfg.linear_key_head_dim,
                 linear_value_head_dim=cfg.linear_value_head_dim,
                 linear_conv_kernel_dim=cfg.linear_conv_kernel,
                 num_experts=cfg.num_experts, num_experts_per_tok=cfg.topk,
                 moe_intermediate_size=cfg.moe_intermediate_size,
                 shared_expert_intermediate_size=cfg.shared_expert_intermediate_size,
                 partial_rotary_factor=cfg.partial_rotary_factor, norm_topk_prob=cfg.norm_topk_prob,
                 decoder_sparse_step=cfg.moe_layer_freq, mlp_only_layers=[],
                 layer_types=["linear_attention" if cfg.layer_is_linear(i) else "full_attention"
                              for i in range(cfg.num_layers)])
        d["rope_parameters"]["partial_rotary_factor"] = cfg.partial_rotary_factor
    elif cfg.arch in ("qwen2", "llama", "mistral"):
        cls = {"qwen2": "Qwen2ForCausalLM", "llama": "LlamaForCausalLM", "mistral": "MistralForCausalLM"}
        d.update(model_type=cfg.arch, architectures=[cls[cfg.arch]])
        if cfg.arch != "qwen2":
            d.update(attention_bias=cfg.attention_bias, mlp_bias=False)
    else:
        d.update(model_type="qwen3", architectures=["Qwen3ForCausalLM"])
    if cfg.mtp_num_layers:
        d["num_nextn_predict_layers"] = cfg.mtp_num_layers
    return d


def save_hf(model: Transformer, path: str, max_shard_bytes: int = 5 << 30) -> None:
    os.makedirs(path, exist_ok=True)
    if hasattr(model, "_sync_fp32"):  # fp32-pinned copies take the latest update first
        model._sync_fp32()
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(hf_config_dict(model.cfg), f, indent=2)
    shard, size, idx, weight_map = {}, 0, 0, {}
    total = 0

    def flush():
        nonlocal shard, size, idx
        if not shard:
            return
        idx += 1
        fn = (f"model-{idx:05d}.safetensors" if stage is None else f"model-pp{stage:02d}-{idx:05d}.safetensors")
        if ep is not None:
            fn = fn.replace("model-", f"model-ep{ep.rank:02d}-")
        save_file(shard, os.path.join(path, fn), metadata={"format": "pt"})
        for n in shard:
            weight_map[n] = fn
        shard, size = {}, 0

    # tensor parallel: every TP rank takes part in the gathers, TP rank 0 writes;
    # pipeline parallel: every stage writes its own files, stage 0 writes the merged index;
    # expert parallel: every EP rank writes its experts, EP rank 0 the rest and the index
    writer = model.tp is None or model.tp.rank == 0
    stage = model.pp.stage if model.pp is not None else None
    ep = getattr(model, "ep", None)
    if stage is not None and stage > 0 and model.cfg.tie_embeddings:
        skip = {"model.embed_tokens.weight"}  # stage 0 writes the tied embedding
    else:
        skip = set()
    if ep is not None:
        import torch.distributed as dist

        ep_first = 0 in dist.get_process_group_ranks(ep.group)  # the EP group rank 0 is in
    for name, t in to_hf_tensors(model):
        tpc = model_tp(model, name)
        internal = name[len("model."):] if name.startswith("model.") else name
        if internal in getattr(model, "fp32", {}):  # fp32-pinned: export the fp32 value
            t = model.fp32[internal]
        t = tp_gather_for(model, name, t.detach())
        if name in skip:
            continue
        if ep is not None and ".mlp.experts." in name:
            # experts: every EP rank of the first EP group (TP rank 0 when TP splits them)
            if not ep_first or (tpc is not None and tpc.rank != 0):
                continue
        elif not writer or (ep is not None and ep.rank != 0):
            continue
        t = to_hf_layout(model.cfg, name, t)
        if model.cfg.arch == "qwen3_5" and name.startswith("model."):
            name = "model.language_model." + name[len("model."):]  # the layout HF Qwen3.5 reads
        t = t.to("cpu").contiguous().clone()
        nb = t.numel() * t.element_size()
        if size + nb > max_shard_bytes:
            flush()
        shard[name] = t
        size += nb
        total += nb
    flush()
    if ep is not None:
        import torch.distributed as dist

        parts: list = [None] * ep.size
        dist.all_gather_object(parts, (weight_map, total), group=ep.group)
        if dist.get_rank() != 0:
            return
        weight_map, total = {}, 0
        for wm, tt in parts:
            weight_map.update(wm)
            total += tt
    if model.pp is not None:
        import torch.distributed as dist

        parts: list = [None] * model.pp.size
        dist.all_gather_object(parts, (weight_map, total), group=model.pp.group)
        if stage != 0:
            return
        weight_map, total = {}, 0
        for wm, tt in parts:
            weight_map.update(wm)
            total += tt
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)


def _open_all(path: str) -> dict[str, str]:
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            return json.load(f)["weight_map"]
    files = [f for f in os.listdir(path) if f.endswith(".safetensors")]
    m = {}
    for fn in files:
        with safe_open(os.path.join(path, fn), "pt") as f:
            for k in f.keys():
                m[k] = fn
    return m


@torch.no_grad()
def load_hf(model: Transformer, path: str) -> None:
    """Load an HF checkpoint into the flat parameter buffer (joins fused projections)."""
    wmap = _open_all(path)
    handles: dict[str, object] = {}

    def get(name):
        fn = wmap[name]
        if fn not in handles:
            handles[fn] = safe_open(os.path.join(path, fn), "pt")
        return handles[fn].get_tensor(name)

    _load(model, wmap, get, path)


@torch.no_grad()
def load_hf_tensors(model: Transformer, tensors: dict[str, torch.Tensor]) -> None:
    """Load HF-named tensors held in memory (e.g. gathered from an FSDP-trained HF model)."""
    _load(model, tensors, tensors.__getitem__, "the given tensors")


def _load(model: Transformer, wmap, get, path: str) -> None:
    cfg = model.cfg
    model._fp8_version = None  # new weights: the fp8 copies (if any) re-quantise on next use
    model._qat_version = None

    targets = dict(to_hf_tensors(model))  # views into model.flat
    missing_mtp: list[str] = []
    for name, dst in targets.items():
        src_name = name
        if src_name not in wmap and src_name.startswith("model.") is False and ("model." + src_name) in wmap:
            src_name = "model." + src_name
        if src_name not in wmap and name.startswith("model."):
            # multimodal checkpoints (Qwen3.5) keep the text model under model.language_model.
            alt = "model.language_model." + name[len("model."):]
            if alt in wmap:
                src_name = alt
        if src_name not in wmap:
            if name == "lm_head.weight" and cfg.tie_embeddings:
                continue
            if _is_mtp_name(model, name):
                # a base checkpoint without multi-token prediction weights: keep the freshly
                # initialised MTP parameters
                missing_mtp.append(name)
                continue
            raise KeyError(f"{name} missing from {path}")
        src = from_hf_layout(cfg, name, get(src_name))
        dst.copy_(tp_slice_for(model, name, src).to(dst.dtype))
        internal = name[len("model."):] if name.startswith("model.") else name
        if internal in getattr(model, "fp32", {}):  # keep the checkpoint's full precision
            model.set_fp32_value(internal, tp_slice_for(model, name, src))
    if missing_mtp:
        warnings.warn(f"{path} has no multi-token prediction weights ({len(missing_mtp)} tensors, "
                      f"e.g. {missing_mtp[0]}); keeping the initialised MTP layers")


def _is_mtp_name(model: Transformer, name: str) -> bool:
    """True for a tensor of a multi-token prediction depth (layers numbered past the main stack)."""
    mtp = set(getattr(model, "mtp_ids", []))
    if not mtp:
        return False
    parts = name.split(".")
    for a, b in zip(parts, parts[1:]):
        if a == "layers" and b.isdigit():
            return int(b) in mtp
    return False
