"""fp32 pinning of marked parameters: a bf16 model keeps the router's expert-score bias and
Gated DeltaNet's A_log / dt_bias at the checkpoint's fp32 values at runtime (the forward reads the
fp32 copy, the HF export writes it back), gradients still reach the bf16 parameters, and a
training update of a pinned parameter replaces its fp32 value."""
import torch

from miles_b200.checkpoint.hf import load_hf, save_hf
from miles_b200.models.config import preset
from miles_b200.models.transformer import Transformer


def test_router_bias_and_gdn_params_stay_fp32(tmp_path):
    from safetensors import safe_open
    from safetensors.torch import load_file, save_file

    for name, key in (("tiny-mla", "layers.1.mlp.gate.e_score_correction_bias"),
                      ("tiny-gdn", "layers.0.linear_attn.A_log")):
        cfg = preset(name)
        src = Transformer(cfg, device="cpu", dtype=torch.float32, seed=0)
        d = str(tmp_path / name)
        save_hf(src, d)
        # give the pinned tensor values that bf16 cannot hold
        fn = [f for f in __import__("os").listdir(d) if f.endswith(".safetensors")][0]
        sd = load_file(f"{d}/{fn}")
        hf_key = "model." + key
        sd[hf_key] = torch.linspace(-1.0, 1.0, sd[hf_key].numel()).float() + 1e-4
        save_file(sd, f"{d}/{fn}")
        m = Transformer(cfg, device="cpu", dtype=torch.bfloat16, seed=1)
        load_hf(m, d)
        want = sd[hf_key]
        assert torch.equal(m.fp32[key], want)
        assert not torch.equal(m.params[key].float(), want)  # the bf16 buffer rounds
        with torch.no_grad():
            assert torch.equal(m.pinned_param(key), want)
        out = str(tmp_path / (name + "_out"))
        save_hf(m, out)
        with safe_open(f"{out}/{[f for f in __import__('os').listdir(out) if f.endswith('.safetensors')][0]}", "pt") as f:
            assert torch.equal(f.get_tensor(hf_key), want)
        # gradient reaches the bf16 parameter; an update replaces the fp32 value
        p = m.params[key]
        v = m.pinned_param(key)
        (v * torch.arange(v.numel())).sum().backward()
        assert p.grad is not None and torch.equal(p.grad.float(), torch.arange(v.numel()).float())
        with torch.no_grad():
            p.add_(1.0)
        m.weight_version += 1
        m.sync_fp8()
        assert torch.equal(m.fp32[key], p.detach().float())
