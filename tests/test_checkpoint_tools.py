"""Checkpoint formats and converters on CPU: HF export/import round trip, torch_dist (DCP)
round trip with Megatron key names, quantized HF exports."""
import json
import os

import torch

from miles_b200.checkpoint.hf import load_hf, save_hf
from miles_b200.checkpoint.torch_dist import load_checkpoint, model_state_dict, save_checkpoint
from miles_b200.models.config import preset
from miles_b200.models.transformer import Transformer
from miles_b200.tools.convert import main as convert


def _m(name="tiny-moe", seed=0):
    return Transformer(preset(name), device="cpu", dtype=torch.float32, seed=seed)


def test_hf_roundtrip(tmp_path):
    a = _m()
    save_hf(a, str(tmp_path / "hf"))
    cfg = json.load(open(tmp_path / "hf" / "config.json"))
    assert cfg["model_type"] == "qwen3_moe" and cfg["num_experts"] == 8
    b = _m(seed=1)
    load_hf(b, str(tmp_path / "hf"))
    assert torch.equal(a.flat, b.flat)


def test_torch_dist_roundtrip(tmp_path):
    a = _m()
    sd = model_state_dict(a)
    assert "decoder.layers.0.self_attention.linear_qkv.weight" in sd
    assert "decoder.layers.1.mlp.experts.linear_fc1.weight" in sd
    save_checkpoint(str(tmp_path / "ck"), 7, a, None, save_optim=False)
    assert open(tmp_path / "ck" / "latest_checkpointed_iteration.txt").read() == "7"
    b = _m(seed=3)
    info = load_checkpoint(str(tmp_path / "ck"), b, None, load_optim=False)
    assert info["iteration"] == 7 and torch.equal(a.flat, b.flat)


def test_quantized_exports(tmp_path):
    a = Transformer(preset("tiny"), device="cpu", dtype=torch.bfloat16, seed=0)
    save_hf(a, str(tmp_path / "hf"))
    for cmd in ("hf2fp8", "hf2int4", "hf2nvfp4", "hf2mxfp8"):
        out = tmp_path / cmd
        convert([cmd, "--hf", str(tmp_path / "hf"), "--out", str(out), "--device", "cpu"])
        cfg = json.load(open(out / "config.json"))
        assert "quantization_config" in cfg
        assert any(f.endswith(".safetensors") for f in os.listdir(out))
    convert(["fp8tobf16", "--hf", str(tmp_path / "hf2fp8"), "--out", str(tmp_path / "back"), "--device", "cpu"])
