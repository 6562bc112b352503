"""Model math and checkpoint mapping against the HuggingFace transformers implementations
(CPU, fp32, tiny random configs): HF model -> save_pretrained -> our load_hf gives the same
logits, and our save_hf -> HF from_pretrained gives them back (Qwen3 dense, Qwen3-MoE,
DeepSeek-V3 MLA + grouped sigmoid MoE with interleaved rotary)."""
import os

import pytest
import torch

os.environ.setdefault("MILES_B200_FORCE_CPU", "1")
transformers = pytest.importorskip("transformers")


def _models():
    from transformers import (DeepseekV3Config, DeepseekV3ForCausalLM, Qwen3Config, Qwen3ForCausalLM,
                              Qwen3MoeConfig, Qwen3MoeForCausalLM)

    yield "qwen3", Qwen3ForCausalLM, Qwen3Config(
        vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, tie_word_embeddings=True,
        rope_theta=1e6)
    yield "qwen3_moe", Qwen3MoeForCausalLM, Qwen3MoeConfig(
        vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        num_experts=8, num_experts_per_tok=2, norm_topk_prob=True)
    yield "deepseek_v3", DeepseekV3ForCausalLM, DeepseekV3Config(
        vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4, n_routed_experts=8,
        num_experts_per_tok=2, n_shared_experts=1, first_k_dense_replace=1, n_group=2, topk_group=1,
        routed_scaling_factor=2.5, kv_lora_rank=64, q_lora_rank=96, qk_nope_head_dim=32,
        qk_rope_head_dim=16, v_head_dim=32, tie_word_embeddings=False)


@pytest.mark.parametrize("name", ["qwen3", "qwen3_moe", "deepseek_v3"])
def test_matches_transformers(tmp_path, name):
    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    _, cls, hcfg = next(x for x in _models() if x[0] == name)
    torch.manual_seed(0)
    hf = cls(hcfg).eval()
    with torch.no_grad():  # non-trivial router correction biases
        for mod in hf.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.1)
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 29))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        h = m.forward_train(toks[0].int(), VarlenMeta([0, 29], "cpu"))
        ours = h.float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())
    # export: our checkpoint loads into transformers and gives the same logits
    save_hf(m, str(tmp_path / "ours"))
    hf2 = cls.from_pretrained(str(tmp_path / "ours"), torch_dtype=torch.float32).eval()
    with torch.no_grad():
        back = hf2(toks).logits[0].float()
    assert (back - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())


def test_qwen3_next_matches_transformers(tmp_path):
    """Qwen3-Next hybrid: Gated DeltaNet layers (HF's torch fallback of the chunked gated delta
    rule), gated full attention with partial rotary, zero-centred norms, MoE with a gated shared
    expert."""
    from transformers import Qwen3NextConfig, Qwen3NextForCausalLM

    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    hc = Qwen3NextConfig(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                         shared_expert_intermediate_size=192, num_hidden_layers=4, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=128, num_experts=8, num_experts_per_tok=2,
                         linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32,
                         linear_value_head_dim=32, linear_conv_kernel_dim=4, full_attention_interval=4,
                         decoder_sparse_step=1, norm_topk_prob=True, tie_word_embeddings=False)
    hf = Qwen3NextForCausalLM(hc).eval()
    with torch.no_grad():  # non-trivial zero-centred norm offsets and decays
        for n, p in hf.named_parameters():
            if n.endswith(("layernorm.weight", "q_norm.weight", "k_norm.weight", "model.norm.weight")):
                p.normal_(0, 0.1)
            if n.endswith("A_log"):
                p.uniform_(-1, 1)
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    assert cfg.layer_is_linear(0) and not cfg.layer_is_linear(3) and cfg.partial_rotary_factor == 0.25
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 37))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        h = m.forward_train(toks[0].int(), VarlenMeta([0, 37], "cpu"))
        ours = h.float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item()), (ref - ours).abs().max()
    save_hf(m, str(tmp_path / "ours"))
    hf2 = Qwen3NextForCausalLM.from_pretrained(str(tmp_path / "ours"), torch_dtype=torch.float32).eval()
    with torch.no_grad():
        back = hf2(toks).logits[0].float()
    assert (back - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())


def test_glm5_dsa_matches_transformers(tmp_path):
    """GLM-5 (DSA): MLA + lightning indexer top-k sparse attention + grouped sigmoid MoE, with
    sequences longer than index_topk so the key selection is active."""
    from transformers import GlmMoeDsaConfig, GlmMoeDsaForCausalLM

    from miles_b200.checkpoint.hf import load_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    hc = GlmMoeDsaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                         num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=4,
                         n_routed_experts=8, num_experts_per_tok=2, n_shared_experts=1, n_group=1,
                         topk_group=1, routed_scaling_factor=2.5, kv_lora_rank=64, q_lora_rank=96,
                         qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32, index_n_heads=16,
                         index_head_dim=32, index_topk=12, mlp_layer_types=["dense", "sparse"],
                         tie_word_embeddings=False)
    # eager attention: transformers' SDPA path for this model combines the index mask with no
    # causal mask when it has none to pass (non-causal attention)
    hc._attn_implementation = "eager"
    hf = GlmMoeDsaForCausalLM(hc).eval()
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    assert cfg.index_topk == 12 and cfg.first_k_dense == 1
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 40))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        h = m.forward_train(toks[0].int(), VarlenMeta([0, 40], "cpu"))
        ours = h.float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item()), (ref - ours).abs().max()


def test_glm45_moe_matches_transformers(tmp_path):
    """GLM-4.5 (glm4_moe): attention with q/k/v biases, QK-norm and half-width rotary; grouped
    sigmoid MoE with a shared expert after one dense layer."""
    from transformers import Glm4MoeConfig, Glm4MoeForCausalLM

    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    hc = Glm4MoeConfig(vocab_size=512, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
                       num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                       n_routed_experts=8, num_experts_per_tok=2, n_shared_experts=1, first_k_dense_replace=1,
                       n_group=2, topk_group=1, routed_scaling_factor=2.5, attention_bias=True,
                       use_qk_norm=True, partial_rotary_factor=0.5, tie_word_embeddings=False)
    hf = Glm4MoeForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if n.endswith("_proj.bias"):
                p.normal_(0, 0.1)
        for mod in hf.modules():
            if hasattr(mod, "e_score_correction_bias"):
                mod.e_score_correction_bias.normal_(0, 0.1)
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    assert cfg.attention_bias and cfg.partial_rotary_factor == 0.5 and cfg.uses_torch_attention
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 33))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        h = m.forward_train(toks[0].int(), VarlenMeta([0, 33], "cpu"))
        ours = h.float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item()), (ref - ours).abs().max()
    save_hf(m, str(tmp_path / "ours"))
    hf2 = Glm4MoeForCausalLM.from_pretrained(str(tmp_path / "ours"), torch_dtype=torch.float32).eval()
    with torch.no_grad():
        back = hf2(toks).logits[0].float()
    assert (back - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("name", ["qwen2", "llama3"])
def test_dense_classics_match_transformers(tmp_path, name):
    """Qwen2.5 (q/k/v biases, no QK-norm) and Llama 3.1 (frequency-band rotary scaling)."""
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen2Config, Qwen2ForCausalLM

    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    if name == "qwen2":
        cls = Qwen2ForCausalLM
        hf = cls(Qwen2Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                             num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=True)).eval()
        with torch.no_grad():
            for n, p in hf.named_parameters():
                if n.endswith("bias"):
                    p.normal_(0, 0.1)
    else:
        cls = LlamaForCausalLM
        hf = cls(LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                             num_attention_heads=4, num_key_value_heads=2,
                             rope_parameters={"rope_type": "llama3", "rope_theta": 500000.0, "factor": 8.0,
                                              "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                              "original_max_position_embeddings": 64})).eval()
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 31))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        ours = m.forward_train(toks[0].int(), VarlenMeta([0, 31], "cpu")).float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())
    save_hf(m, str(tmp_path / "ours"))
    with torch.no_grad():
        back = cls.from_pretrained(str(tmp_path / "ours"), torch_dtype=torch.float32).eval()(toks).logits[0].float()
    assert (back - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())


def test_qwen35_moe_matches_transformers(tmp_path):
    """Qwen3.5 MoE (text): the Qwen3-Next hybrid with separate in_proj_qkv / z / b / a."""
    from transformers import Qwen3_5MoeForCausalLM, Qwen3_5MoeTextConfig

    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    hc = Qwen3_5MoeTextConfig(vocab_size=512, hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                              num_key_value_heads=2, head_dim=128, linear_num_key_heads=2,
                              linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
                              moe_intermediate_size=128, shared_expert_intermediate_size=192, num_experts=8,
                              num_experts_per_tok=2, tie_word_embeddings=False,
                              layer_types=["linear_attention"] * 3 + ["full_attention"])
    hf = Qwen3_5MoeForCausalLM(hc).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if n.endswith(("layernorm.weight", "q_norm.weight", "k_norm.weight", "model.norm.weight")):
                p.normal_(0, 0.1)
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    assert cfg.arch == "qwen3_5" and cfg.layer_is_linear(2) and not cfg.layer_is_linear(3)
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 29))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        ours = m.forward_train(toks[0].int(), VarlenMeta([0, 29], "cpu")).float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item()), (ref - ours).abs().max()
    save_hf(m, str(tmp_path / "ours"))
    with torch.no_grad():
        back = Qwen3_5MoeForCausalLM.from_pretrained(str(tmp_path / "ours"),
                                                     torch_dtype=torch.float32).eval()(toks).logits[0].float()
    assert (back - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())


def test_glm4_dense_matches_transformers(tmp_path):
    """GLM-4 dense: sandwich norms, adjacent-pair half-width rotary, q/k/v biases, fused gate_up."""
    from transformers import Glm4Config, Glm4ForCausalLM

    from miles_b200.checkpoint.hf import load_hf, save_hf
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    hf = Glm4ForCausalLM(Glm4Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                    num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                    tie_word_embeddings=False, pad_token_id=0)).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if n.endswith("bias"):
                p.normal_(0, 0.1)
            if n.endswith("layernorm.weight"):
                p.normal_(1.0, 0.1)
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    assert cfg.sandwich_norm and cfg.rope_interleave
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    toks = torch.randint(0, cfg.vocab_size, (1, 27))
    with torch.no_grad():
        ref = hf(toks).logits[0].float()
        ours = m.forward_train(toks[0].int(), VarlenMeta([0, 27], "cpu")).float() @ m.lm_head_weight().float().t()
    assert (ref - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item()), (ref - ours).abs().max()
    save_hf(m, str(tmp_path / "ours"))
    with torch.no_grad():
        back = Glm4ForCausalLM.from_pretrained(str(tmp_path / "ours"), torch_dtype=torch.float32).eval()(toks).logits[0].float()
    assert (back - ours).abs().max() < 1e-4 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("family", ["qwen2", "glm4", "glm45", "qwen3_next"])
def test_engine_decode_matches_forward_for_hf_families(tmp_path, family):
    """The rollout engine's prefill + decode path (paged cache, separate-projection attention,
    sandwich norms, gated attention / GDN state) reproduces the training forward."""
    import numpy as np
    from transformers import (Glm4Config, Glm4ForCausalLM, Glm4MoeConfig, Glm4MoeForCausalLM, Qwen2Config,
                              Qwen2ForCausalLM, Qwen3NextConfig, Qwen3NextForCausalLM)

    from miles_b200.checkpoint.hf import load_hf
    from miles_b200.engine.engine import GenRequest, RolloutEngine
    from miles_b200.models.config import ModelConfig
    from miles_b200.models.transformer import Transformer
    from miles_b200.ops.attention import VarlenMeta

    torch.manual_seed(0)
    base = dict(vocab_size=512, hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                num_key_value_heads=2, tie_word_embeddings=False)
    if family == "qwen2":
        hf = Qwen2ForCausalLM(Qwen2Config(intermediate_size=512, **base))
    elif family == "glm4":
        hf = Glm4ForCausalLM(Glm4Config(intermediate_size=512, head_dim=64, pad_token_id=0, **base))
    elif family == "glm45":
        hf = Glm4MoeForCausalLM(Glm4MoeConfig(intermediate_size=512, moe_intermediate_size=128, head_dim=64,
                                              n_routed_experts=8, num_experts_per_tok=2, first_k_dense_replace=1,
                                              attention_bias=True, use_qk_norm=True, **base))
    else:
        hf = Qwen3NextForCausalLM(Qwen3NextConfig(intermediate_size=512, moe_intermediate_size=128,
                                                  shared_expert_intermediate_size=128, head_dim=128,
                                                  num_experts=8, num_experts_per_tok=2, linear_num_key_heads=2,
                                                  linear_num_value_heads=4, linear_key_head_dim=32,
                                                  linear_value_head_dim=32, full_attention_interval=2, **base))
    hf.save_pretrained(str(tmp_path / "hf"))
    cfg = ModelConfig.from_hf(str(tmp_path / "hf"))
    m = Transformer(cfg, device="cpu", dtype=torch.float32, seed=1)
    load_hf(m, str(tmp_path / "hf"))
    eng = RolloutEngine(m, max_batch=2, num_pages=32, max_pages_per_seq=4, use_cuda_graph=False)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 512, n).tolist() for n in (7, 40, 19)]
    outs = eng.generate([GenRequest(p, 6, temperature=0.0, rid=i) for i, p in enumerate(prompts)])
    for p, o in zip(prompts, outs):
        toks = p + o.tokens
        with torch.no_grad():
            h = m.forward_train(torch.tensor(toks, dtype=torch.int32), VarlenMeta([0, len(toks)], "cpu"))
        logits = h.float() @ m.lm_head_weight().float().t()
        assert logits[len(p) - 1:len(toks) - 1].argmax(-1).tolist() == o.tokens
        lp = torch.log_softmax(logits[len(p) - 1:len(toks) - 1], -1)
        ref = lp.gather(1, torch.tensor(o.tokens)[:, None])[:, 0].detach().numpy()
        assert np.abs(ref - np.asarray(o.logprobs)).max() < 1e-4
