"""Megatron-style `torch_dist` checkpoints (PyTorch Distributed Checkpoint, DCP).

Layout (compatible with the reference's detection rules):
    {save}/latest_checkpointed_iteration.txt          "<iteration>"
    {save}/iter_{iteration:07d}/                      DCP shards (*.distcp, .metadata)
    {save}/iter_{iteration:07d}/common.pt             iteration, rollout id, args, rng
    {save}/rollout/global_dataset_state_dict_{id}.pt  data-source position (written elsewhere)

Parameter keys use Megatron-Core GPT names (decoder.layers.{i}.self_attention.linear_qkv.weight,
...); the fused QKV is stored in Megatron's query-group-interleaved order
([q_g, k_g, v_g] for every KV group g) and converted back on load. Optimizer state (Adam m/v,
fp32 master if present) is saved unless --no-save-optim.

Reference: megatron_utils/checkpoint.py:17-200 (load/save torch_dist, iteration detection
:168-171, HF fallback :174-195), actor.py:469-493 (save_model, async save).
"""
from __future__ import annotations

import os
import re
import threading

import torch
import torch.distributed.checkpoint as dcp

from miles_b200.models.transformer import Transformer

TRACKER = "latest_checkpointed_iteration.txt"


def _qkv_to_megatron(t, nq, nkv, D):
    q, k, v = torch.split(t, [nq * D, nkv * D, nkv * D], 0)
    G = nq // nkv
    q = q.view(nkv, G * D, -1)
    k = k.view(nkv, D, -1)
    v = v.view(nkv, D, -1)
    return torch.cat([q, k, v], 1).reshape(t.shape)


def _qkv_from_megatron(t, nq, nkv, D):
    G = nq // nkv
    x = t.view(nkv, (G + 2) * D, -1)
    q, k, v = torch.split(x, [G * D, D, D], 1)
    return torch.cat([q.reshape(nq * D, -1), k.reshape(nkv * D, -1), v.reshape(nkv * D, -1)], 0)


class _NoMTP:
    """cfg view whose main stack covers every layer index (names an MTP layer's body)."""

    def __init__(self, cfg):
        self._c = cfg

    def __getattr__(self, k):
        return 1 << 30 if k == "num_layers" else getattr(self._c, k)


def megatron_name(name: str, cfg) -> str:
    m = re.match(r"layers\.(\d+)\.(.*)", name)
    if not m:
        return {"embed_tokens.weight": "embedding.word_embeddings.weight",
                "norm.weight": "decoder.final_layernorm.weight",
                "lm_head.weight": "output_layer.weight"}[name]
    i, rest = int(m.group(1)), m.group(2)
    L = f"decoder.layers.{i}."
    if i >= cfg.num_layers:  # multi-token prediction depth (Megatron MTP block names)
        mp = f"mtp.layers.{i - cfg.num_layers}."
        extra = {"enorm.weight": "enorm.weight", "hnorm.weight": "hnorm.weight",
                 "eh_proj.weight": "eh_proj.weight", "shared_head.norm.weight": "final_layernorm.weight"}
        if rest in extra:
            return mp + extra[rest]
        return mp + "transformer_layer." + megatron_name(f"layers.{i}.{rest}", _NoMTP(cfg))[len(L):]
    moe = cfg.layer_is_moe(i)
    table = {
        "input_layernorm.weight": ("input_layernorm.weight" if cfg.kv_lora_rank
                                   else "self_attention.linear_qkv.layer_norm_weight"),
        # multi-head latent attention (Megatron MLASelfAttention names)
        "self_attn.q_proj.weight": "self_attention.linear_q_proj.weight",
        "self_attn.q_a_proj.weight": "self_attention.linear_q_down_proj.weight",
        "self_attn.q_a_layernorm.weight": "self_attention.linear_q_up_proj.layer_norm_weight",
        "self_attn.q_b_proj.weight": "self_attention.linear_q_up_proj.weight",
        "self_attn.kv_a_proj_with_mqa.weight": "self_attention.linear_kv_down_proj.weight",
        "self_attn.kv_a_layernorm.weight": "self_attention.linear_kv_up_proj.layer_norm_weight",
        "self_attn.kv_b_proj.weight": "self_attention.linear_kv_up_proj.weight",
        "self_attn.qkv_proj.weight": "self_attention.linear_qkv.weight",
        "self_attn.o_proj.weight": "self_attention.linear_proj.weight",
        "self_attn.q_norm.weight": "self_attention.q_layernorm.weight",
        "self_attn.k_norm.weight": "self_attention.k_layernorm.weight",
        "post_attention_layernorm.weight": "pre_mlp_layernorm.weight" if moe else "mlp.linear_fc1.layer_norm_weight",
        "mlp.gate_up_proj.weight": "mlp.linear_fc1.weight",
        "mlp.down_proj.weight": "mlp.linear_fc2.weight",
        "mlp.gate.weight": "mlp.router.weight",
        "mlp.gate.e_score_correction_bias": "mlp.router.expert_bias",
        "mlp.experts.w1": "mlp.experts.linear_fc1.weight",
        "mlp.experts.w2": "mlp.experts.linear_fc2.weight",
        "mlp.shared_experts.gate_up_proj.weight": "mlp.shared_experts.linear_fc1.weight",
        "mlp.shared_experts.down_proj.weight": "mlp.shared_experts.linear_fc2.weight",
    }
    return L + table[rest]


def _key(model: Transformer, name: str) -> str:
    """Checkpoint key; under tensor parallelism a sharded parameter is stored per TP rank
    (suffix ``.tp<rank>of<size>``), so a torch_dist checkpoint reloads at the same TP size
    (the HF path reshards between sizes)."""
    k = megatron_name(name, model.cfg)
    if model.tp is not None:
        from miles_b200.parallel.tp import is_tp_sharded, model_tp

        if is_tp_sharded(name) and model_tp(model, name) is not None:
            k += f".tp{model.tp.rank}of{model.tp.size}"
    ep = getattr(model, "ep", None)
    if ep is not None and ".mlp.experts." in "." + name:
        k += f".ep{ep.rank}of{ep.size}"  # each EP rank holds a different expert slice
    return k


def model_state_dict(model: Transformer) -> dict[str, torch.Tensor]:
    cfg = model.cfg
    sd = {}
    for name, p in model.params.items():
        t = p.data
        if name.endswith("qkv_proj.weight"):
            t = _qkv_to_megatron(t, model.nq, model.nkv, cfg.head_dim)
        sd[_key(model, name)] = t
    return sd


def get_checkpoint_iteration(load: str) -> int | None:
    p = os.path.join(load, TRACKER)
    if os.path.exists(p):
        with open(p) as f:
            return int(f.read().strip())
    its = [int(m.group(1)) for d in os.listdir(load) if (m := re.fullmatch(r"iter_(\d{7})", d))] \
        if os.path.isdir(load) else []
    return max(its) if its else None


def is_torch_dist(path: str) -> bool:
    return path is not None and os.path.isdir(path) and get_checkpoint_iteration(path) is not None


_ASYNC: threading.Thread | None = None


def _mp_suffix(model) -> str:
    """Key suffix of this rank's model-parallel part (TP rank / pipeline stage / EP rank)."""
    if model is None:
        return ""
    out = ""
    if getattr(model, "tp", None) is not None:
        out += f".tp{model.tp.rank}of{model.tp.size}"
    if getattr(model, "pp", None) is not None:
        v = getattr(model.pp, "vpp", 1)
        out += f".pp{model.pp.stage}of{model.pp.size}" + (f"v{v}" if v > 1 else "")
    if getattr(model, "ep", None) is not None:
        out += f".ep{model.ep.rank}of{model.ep.size}"
    return out


def _optim_state(optimizer, model=None) -> dict:
    """Optimizer tensors under checkpoint keys. A state sharded over data-parallel ranks is
    stored under per-shard keys (each rank writes its own; loading needs the same world), and
    under model parallelism per TP rank / pipeline stage."""
    osd = optimizer.state_dict()
    rank, world = osd.get("shard", (0, 1))
    sfx = (f".shard{rank}of{world}" if world > 1 else "") + _mp_suffix(model)
    out = {"m" + sfx: osd["m"], "v" + sfx: osd["v"]}
    if osd.get("master") is not None:
        out["master" + sfx] = osd["master"]
    return out


def save_checkpoint(save: str, iteration: int, model: Transformer, optimizer=None,
                    extra: dict | None = None, save_optim: bool = True, async_save: bool = False,
                    process_group=None):
    """process_group: the ranks that hold this model (default: the whole world); every one of
    them must call this."""
    global _ASYNC
    d = os.path.join(save, f"iter_{iteration:07d}")
    os.makedirs(d, exist_ok=True)
    sd = {"model": model_state_dict(model)}
    lora = getattr(model, "lora", None)
    if lora is not None:
        # adapters are saved on their own (base weights are frozen); their AdamW state with them
        if not torch.distributed.is_initialized() or torch.distributed.get_rank(process_group) == 0:
            lora.save(os.path.join(d, "lora_adapter.pt"))
            if optimizer is not None and save_optim:
                torch.save(optimizer.state_dict(), os.path.join(d, "lora_optim.pt"))
        save_optim = False
    if optimizer is not None and save_optim:
        sd["optimizer"] = _optim_state(optimizer, model)
    rank0 = not torch.distributed.is_initialized() or torch.distributed.get_rank(process_group) == 0

    def _write(sd_cpu):
        dcp.save(sd_cpu, checkpoint_id=d, process_group=process_group)
        if rank0:
            torch.save({"iteration": iteration, "optimizer_step": getattr(optimizer, "step_id", 0),
                        "weight_version": model.weight_version, "extra": extra or {},
                        "rng": torch.get_rng_state()}, os.path.join(d, "common.pt"))
            with open(os.path.join(save, TRACKER), "w") as f:
                f.write(str(iteration))

    if async_save:
        if _ASYNC is not None:
            _ASYNC.join()
        sd_cpu = {k: ({kk: vv.detach().cpu().clone() for kk, vv in v.items()}) for k, v in sd.items()}
        _ASYNC = threading.Thread(target=_write, args=(sd_cpu,), daemon=True)
        _ASYNC.start()
    else:
        _write(sd)


def wait_async_save():
    if _ASYNC is not None:
        _ASYNC.join()


@torch.no_grad()
def load_checkpoint(load: str, model: Transformer, optimizer=None, load_optim: bool = True,
                    iteration: int | None = None, process_group=None) -> dict:
    it = iteration if iteration is not None else get_checkpoint_iteration(load)
    if it is None:
        raise FileNotFoundError(f"no torch_dist checkpoint under {load}")
    d = os.path.join(load, f"iter_{it:07d}")
    cfg = model.cfg
    model._fp8_version = None  # new weights: the fp8 copies (if any) re-quantise on next use
    model._qat_version = None
    sd = {"model": {k: torch.empty_like(v) for k, v in model_state_dict(model).items()}}
    lora = getattr(model, "lora", None)
    if lora is not None:
        if os.path.exists(os.path.join(d, "lora_adapter.pt")):
            lora.load(os.path.join(d, "lora_adapter.pt"))
        if optimizer is not None and load_optim and os.path.exists(os.path.join(d, "lora_optim.pt")):
            optimizer.load_state_dict(torch.load(os.path.join(d, "lora_optim.pt"), weights_only=False))
        load_optim = False
    if optimizer is not None and load_optim:
        sd["optimizer"] = _optim_state(optimizer, model)  # views of the live state: loaded in place
    dcp.load(sd, checkpoint_id=d, process_group=process_group)
    for name, p in model.params.items():
        t = sd["model"][_key(model, name)]
        if name.endswith("qkv_proj.weight"):
            t = _qkv_from_megatron(t, model.nq, model.nkv, cfg.head_dim)
        p.data.copy_(t)
    common = torch.load(os.path.join(d, "common.pt"), weights_only=False) if os.path.exists(os.path.join(d, "common.pt")) else {}
    if optimizer is not None and load_optim:
        optimizer.step_id = common.get("optimizer_step", 0)
    model.weight_version = common.get("weight_version", 0)
    return {"iteration": it, **common}
