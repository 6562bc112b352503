"""Model configurations: HF-config parsing plus the presets the benchmarks name.

Reference: model shapes from scripts/models/*.sh (e.g. qwen3-30B-A3B.sh, qwen3-4B.sh) and the
HF configs the reference's mbridge / megatron_to_hf converters read.
"""
from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field


@dataclass
class ModelConfig:
    arch: str = "qwen3"               # qwen3 | qwen3_moe | deepseek_v3
    vocab_size: int = 151936
    hidden_size: int = 2048
    num_layers: int = 2
    num_heads: int = 16
    num_kv_heads: int = 4
    head_dim: int = 128
    intermediate_size: int = 6144     # dense FFN
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    rope_scaling: dict | None = None
    max_position: int = 40960
    tie_embeddings: bool = False
    qk_norm: bool = True
    # MoE
    num_experts: int = 0
    topk: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    router_score: str = "softmax"     # softmax | sigmoid
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    num_shared_experts: int = 0
    first_k_dense: int = 0            # leading dense layers (DeepSeek)
    mtp_num_layers: int = 0           # multi-token prediction depths (layers num_layers .. + mtp - 1)
    moe_layer_freq: int = 1
    # MLA (DeepSeek-V3 style)
    kv_lora_rank: int = 0
    q_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0
    rope_interleave: bool = False  # MLA rotary dims stored as interleaved pairs (DeepSeek-V3 HF)
    # DSA (DeepSeek-V3.2 / GLM-5 sparse attention): lightning indexer + top-k key selection
    index_n_heads: int = 0
    index_head_dim: int = 0
    index_topk: int = 0
    # Gated DeltaNet hybrid (Qwen3-Next): every `linear_attn_interval`-th layer keeps softmax
    # attention, the others are linear attention (0 = no linear layers)
    linear_attn_interval: int = 0
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel: int = 4
    # Qwen3-Next full-attention layers: output gate, partial rotary; MoE shared expert with a gate
    attn_output_gate: bool = False
    partial_rotary_factor: float = 1.0
    norm_offset: bool = False          # checkpoint RMSNorm weights are w in y = x_hat * (1 + w)
    shared_expert_intermediate_size: int = 0
    attention_bias: bool = False       # q / k / v projection biases (GLM-4.5)
    sandwich_norm: bool = False        # GLM-4: RMSNorm on the attention and MLP outputs as well
    extra: dict = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def uses_torch_attention(self) -> bool:
        """Softmax attention with an output gate, projection biases or partial rotary: the
        separate q / k / v projection path of models/qwen3_next.py instead of the fused
        qkv + QK-norm/RoPE kernel."""
        return (self.attn_output_gate or self.attention_bias or self.partial_rotary_factor != 1.0
                or (self.rope_interleave and not self.kv_lora_rank))

    def layer_is_linear(self, i: int) -> bool:
        # layers numbered past the main stack are multi-token prediction depths: full attention
        return (self.linear_attn_interval > 0 and i < self.num_layers
                and (i + 1) % self.linear_attn_interval != 0)

    def layer_is_moe(self, i: int) -> bool:
        return self.is_moe and i >= self.first_k_dense and (i - self.first_k_dense) % self.moe_layer_freq == 0

    def num_params(self) -> int:
        H, D = self.hidden_size, self.head_dim
        attn = H * (self.num_heads + 2 * self.num_kv_heads) * D + self.num_heads * D * H + 2 * H + 2 * D
        n = 0
        for i in range(self.num_layers):
            n += attn
            if self.layer_is_moe(i):
                n += self.num_experts * 3 * H * self.moe_intermediate_size + self.num_experts * H
                n += self.num_shared_experts * 3 * H * self.moe_intermediate_size
            else:
                n += 3 * H * self.intermediate_size
        n += self.vocab_size * H * (1 if self.tie_embeddings else 2) + H
        return n

    def active_params(self) -> int:
        """Parameters touched per token (for FLOP accounting)."""
        H, D = self.hidden_size, self.head_dim
        attn = H * (self.num_heads + 2 * self.num_kv_heads) * D + self.num_heads * D * H
        n = 0
        for i in range(self.num_layers):
            n += attn
            if self.layer_is_moe(i):
                n += (self.topk + self.num_shared_experts) * 3 * H * self.moe_intermediate_size
            else:
                n += 3 * H * self.intermediate_size
        return n + self.vocab_size * H

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_hf(cls, path_or_dict) -> "ModelConfig":
        if isinstance(path_or_dict, str):
            p = path_or_dict
            if os.path.isdir(p):
                p = os.path.join(p, "config.json")
            with open(p) as f:
                d = json.load(f)
        else:
            d = dict(path_or_dict)
        mt = d.get("model_type", "qwen3")
        c = cls()
        c.vocab_size = d["vocab_size"]
        c.hidden_size = d["hidden_size"]
        c.num_layers = d["num_hidden_layers"]
        c.num_heads = d["num_attention_heads"]
        c.num_kv_heads = d.get("num_key_value_heads", c.num_heads)
        c.head_dim = d.get("head_dim", c.hidden_size // c.num_heads)
        c.intermediate_size = d.get("intermediate_size", 0)
        c.rms_eps = d.get("rms_norm_eps", 1e-6)
        # transformers >= 5 nests the rotary settings in `rope_parameters`
        rp = d.get("rope_parameters") or {}
        c.rope_theta = d.get("rope_theta", rp.get("rope_theta", 1e4))
        c.rope_scaling = d.get("rope_scaling")
        if c.rope_scaling is None and rp.get("rope_type", "default") not in ("default", None):
            c.rope_scaling = {k: v for k, v in rp.items() if k != "rope_theta"}
        c.max_position = d.get("max_position_embeddings", 32768)
        c.tie_embeddings = d.get("tie_word_embeddings", False)
        c.extra["token_ids"] = {k: d.get(k) for k in ("pad_token_id", "bos_token_id", "eos_token_id")}
        c.extra["num_nextn_predict_layers"] = int(d.get("num_nextn_predict_layers") or 0)
        if mt == "glm4":  # GLM-4 dense: sandwich norms, interleaved half-width rotary, biases
            c.arch = "glm4"
            c.sandwich_norm = True
            c.rope_interleave = True
            c.qk_norm = False
            c.attention_bias = bool(d.get("attention_bias", True))
            c.partial_rotary_factor = d.get("partial_rotary_factor", rp.get("partial_rotary_factor", 0.5))
            return c
        if mt == "glm4_moe":  # GLM-4.5: GQA with biases / partial rotary, DeepSeek-style MoE
            c.arch = "glm4_moe"
            c.num_experts = d["n_routed_experts"]
            c.topk = d["num_experts_per_tok"]
            c.moe_intermediate_size = d["moe_intermediate_size"]
            c.num_shared_experts = d.get("n_shared_experts", 0)
            c.first_k_dense = d.get("first_k_dense_replace", 0)
            c.router_score = "sigmoid"
            c.n_group = d.get("n_group", 1)
            c.topk_group = d.get("topk_group", 1)
            c.routed_scaling_factor = d.get("routed_scaling_factor", 1.0)
            c.norm_topk_prob = d.get("norm_topk_prob", True)
            c.attention_bias = bool(d.get("attention_bias", False))
            c.qk_norm = bool(d.get("use_qk_norm", False))
            c.partial_rotary_factor = d.get("partial_rotary_factor", rp.get("partial_rotary_factor", 1.0))
            return c
        if mt in ("qwen3_next", "qwen3_5_text", "qwen3_5_moe_text"):
            # Qwen3.5 keeps the Qwen3-Next hybrid with separate in_proj_qkv / z / b / a tensors
            c.arch = "qwen3_next" if mt == "qwen3_next" else "qwen3_5"
            c.num_experts = d.get("num_experts", d.get("num_local_experts", 0))
            c.topk = d.get("num_experts_per_tok", 0)
            c.moe_intermediate_size = d.get("moe_intermediate_size", 0)
            c.norm_topk_prob = d.get("norm_topk_prob", True)
            c.linear_attn_interval = d.get("full_attention_interval", 4)
            if "layer_types" in d:
                c.linear_attn_interval = d["layer_types"].index("full_attention") + 1
            c.linear_num_key_heads = d["linear_num_key_heads"]
            c.linear_num_value_heads = d["linear_num_value_heads"]
            c.linear_key_head_dim = d["linear_key_head_dim"]
            c.linear_value_head_dim = d["linear_value_head_dim"]
            c.linear_conv_kernel = d.get("linear_conv_kernel_dim", 4)
            c.intermediate_size = d.get("intermediate_size", 0)
            c.attn_output_gate = True
            c.norm_offset = True
            c.partial_rotary_factor = d.get("partial_rotary_factor", rp.get("partial_rotary_factor", 1.0))
            c.shared_expert_intermediate_size = d.get("shared_expert_intermediate_size", 0)
            c.moe_layer_freq = d.get("decoder_sparse_step", 1)
            return c
        if mt in ("qwen3_moe",):
            c.arch = "qwen3_moe"
            c.num_experts = d.get("num_experts", d.get("num_local_experts"))
            c.topk = d["num_experts_per_tok"]
            c.moe_intermediate_size = d["moe_intermediate_size"]
            c.norm_topk_prob = d.get("norm_topk_prob", True)
        elif mt in ("deepseek_v3", "deepseek_v2", "deepseek_v32", "kimi_k2", "glm4_moe_lite", "glm_moe_dsa"):
            c.arch = "deepseek_v3"
            c.num_experts = d["n_routed_experts"]
            c.topk = d["num_experts_per_tok"]
            c.moe_intermediate_size = d["moe_intermediate_size"]
            c.num_shared_experts = d.get("n_shared_experts", 0)
            c.first_k_dense = d.get("first_k_dense_replace", 0)
            if "mlp_layer_types" in d:  # GLM-5: leading dense layers named per layer
                kinds = d["mlp_layer_types"]
                c.first_k_dense = next((i for i, t in enumerate(kinds) if t == "sparse"), len(kinds))
            c.router_score = d.get("scoring_func", "sigmoid")
            c.n_group = d.get("n_group", 1)
            c.topk_group = d.get("topk_group", 1)
            c.routed_scaling_factor = d.get("routed_scaling_factor", 1.0)
            c.norm_topk_prob = d.get("norm_topk_prob", True)
            c.kv_lora_rank = d.get("kv_lora_rank", 0)
            c.q_lora_rank = d.get("q_lora_rank") or 0
            c.qk_nope_head_dim = d.get("qk_nope_head_dim", 0)
            c.qk_rope_head_dim = d.get("qk_rope_head_dim", 0)
            c.v_head_dim = d.get("v_head_dim", 0)
            c.rope_interleave = bool(d.get("rope_interleave", False))
            c.qk_norm = False
            c.index_n_heads = d.get("index_n_heads", 0)
            c.index_head_dim = d.get("index_head_dim", 0)
            c.index_topk = d.get("index_topk", 0)
        else:
            c.arch = "qwen3" if mt == "qwen3" else mt
            c.qk_norm = mt == "qwen3"
            # Qwen2 / Qwen2.5 carry q/k/v biases without a config flag; Llama-style configs say
            c.attention_bias = bool(d.get("attention_bias", mt == "qwen2"))
        return c


def preset(name: str) -> ModelConfig:
    """Named shapes used by the benchmarks and tests (random-init weights)."""
    n = name.lower()
    if n in ("qwen3-30b-a3b", "qwen3_30b_a3b"):
        return ModelConfig(arch="qwen3_moe", vocab_size=151936, hidden_size=2048, num_layers=48,
                           num_heads=32, num_kv_heads=4, head_dim=128, intermediate_size=6144,
                           num_experts=128, topk=8, moe_intermediate_size=768, max_position=40960)
    if n in ("qwen3-4b", "qwen3_4b"):
        return ModelConfig(arch="qwen3", vocab_size=151936, hidden_size=2560, num_layers=36,
                           num_heads=32, num_kv_heads=8, head_dim=128, intermediate_size=9728,
                           tie_embeddings=True)
    if n in ("qwen3-32b", "qwen3_32b"):
        return ModelConfig(arch="qwen3", vocab_size=151936, hidden_size=5120, num_layers=64,
                           num_heads=64, num_kv_heads=8, head_dim=128, intermediate_size=25600)
    if n in ("qwen3-0.6b", "qwen3_0_6b"):
        return ModelConfig(arch="qwen3", vocab_size=151936, hidden_size=1024, num_layers=28,
                           num_heads=16, num_kv_heads=8, head_dim=128, intermediate_size=3072,
                           tie_embeddings=True)
    if n in ("tiny", "tiny-qwen3"):
        # CPU plumbing config: 2 layers, hidden 256, 4q/2kv, head_dim 64, FFN 704, vocab 4096
        return ModelConfig(arch="qwen3", vocab_size=4096, hidden_size=256, num_layers=2,
                           num_heads=4, num_kv_heads=2, head_dim=64, intermediate_size=704,
                           tie_embeddings=True, max_position=4096)
    if n in ("tiny-moe",):
        return ModelConfig(arch="qwen3_moe", vocab_size=4096, hidden_size=256, num_layers=2,
                           num_heads=4, num_kv_heads=2, head_dim=128, num_experts=8, topk=2,
                           moe_intermediate_size=128, max_position=4096)
    if n in ("small-moe",):  # GPU smoke shape (head_dim 128, H multiple of 256)
        return ModelConfig(arch="qwen3_moe", vocab_size=8192, hidden_size=512, num_layers=2,
                           num_heads=8, num_kv_heads=2, head_dim=128, num_experts=16, topk=4,
                           moe_intermediate_size=256, max_position=8192)
    if n in ("tiny-mla",):  # CPU / GPU plumbing shape of the DeepSeek-style MLA + MoE family
        return ModelConfig(arch="deepseek_v3", vocab_size=4096, hidden_size=256, num_layers=2,
                           num_heads=4, num_kv_heads=4, head_dim=128, intermediate_size=512,
                           num_experts=8, topk=2, moe_intermediate_size=128, num_shared_experts=1,
                           first_k_dense=1, router_score="sigmoid", n_group=2, topk_group=1,
                           kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16,
                           v_head_dim=32, qk_norm=False, routed_scaling_factor=2.5,
                           max_position=4096)
    if n in ("tiny-gdn",):  # Gated DeltaNet hybrid: layers 0-2 linear attention, layer 3 softmax
        return ModelConfig(arch="qwen3_next", vocab_size=4096, hidden_size=256, num_layers=4,
                           num_heads=4, num_kv_heads=2, head_dim=128, intermediate_size=512,
                           tie_embeddings=True, max_position=4096, linear_attn_interval=4,
                           linear_num_key_heads=2, linear_num_value_heads=4,
                           linear_key_head_dim=32, linear_value_head_dim=32, attn_output_gate=True,
                           partial_rotary_factor=0.25, norm_offset=True, num_experts=8, topk=2,
                           moe_intermediate_size=128, shared_expert_intermediate_size=192)
    if n in ("tiny-dsa",):  # MLA + lightning indexer with top-k sparse attention (DSA)
        return ModelConfig(arch="deepseek_v3", vocab_size=4096, hidden_size=256, num_layers=2,
                           num_heads=4, num_kv_heads=4, head_dim=128, intermediate_size=512,
                           num_experts=8, topk=2, moe_intermediate_size=128, num_shared_experts=1,
                           first_k_dense=1, router_score="sigmoid", n_group=2, topk_group=1,
                           kv_lora_rank=64, q_lora_rank=96, qk_nope_head_dim=32, qk_rope_head_dim=16,
                           v_head_dim=32, qk_norm=False, routed_scaling_factor=2.5,
                           index_n_heads=4, index_head_dim=32, index_topk=16, max_position=4096)
    if n in ("dsv3-small", "deepseek-v3-small"):
        # DeepSeek-V3-style shape (27 layers): MLA + MoE, sigmoid grouped routing, shared experts
        return ModelConfig(arch="deepseek_v3", vocab_size=163840, hidden_size=2048, num_layers=27,
                           num_heads=16, num_kv_heads=16, head_dim=128, intermediate_size=11264,
                           num_experts=64, topk=6, moe_intermediate_size=1408, num_shared_experts=2,
                           first_k_dense=1, router_score="sigmoid", n_group=1, topk_group=1,
                           kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64,
                           v_head_dim=128, qk_norm=False, routed_scaling_factor=1.0)
    raise KeyError(f"unknown model preset {name!r}")
