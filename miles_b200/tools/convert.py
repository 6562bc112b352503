"""Offline checkpoint converters.

    python -m miles_b200.tools.convert hf2dist  --hf <dir> --save <torch_dist dir> [--model-name preset]
    python -m miles_b200.tools.convert dist2hf  --load <torch_dist dir> --out <hf dir> --hf-config <dir|preset>
    python -m miles_b200.tools.convert hf2fp8   --hf <dir> --out <dir> [--block 128 128] [--ue8m0]
    python -m miles_b200.tools.convert hf2int4  --hf <dir> --out <dir> [--group 128] [--asym]
    python -m miles_b200.tools.convert hf2nvfp4 --hf <dir> --out <dir>
    python -m miles_b200.tools.convert hf2mxfp8 --hf <dir> --out <dir>
    python -m miles_b200.tools.convert fp8tobf16 --hf <dir> --out <dir>

Quantized exports keep norms, embeddings, routers and the LM head in bf16 and write, per
quantized linear weight, the quantized tensor plus its scales (`weight_scale_inv` for fp8
blocks, `weight_scale` / `weight_zero_point` for int4 groups, `weight_scale` +
`weight_scale_2` for NVFP4, `weight_scale` exponents for MXFP8) and a quantization_config in
config.json.

Reference: tools/convert_hf_to_torch_dist.py, convert_torch_dist_to_hf.py,
convert_hf_to_fp8.py, convert_hf_to_int4*.py, convert_hf_to_nvfp4.py, convert_hf_to_mxfp8.py,
fp8_cast_bf16.py.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from miles_b200.ops import quant as Q

SKIP = ("norm", "embed_tokens", "lm_head", "mlp.gate.", "e_score_correction_bias")


def _quantizable(name: str, t: torch.Tensor) -> bool:
    return name.endswith(".weight") and t.dim() == 2 and not any(s in name for s in SKIP)


def _iter_hf(path):
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    for fn in files:
        with safe_open(os.path.join(path, fn), "pt") as f:
            for k in f.keys():
                yield fn, k, f.get_tensor(k)


def _copy_meta(src, dst, qcfg=None):
    os.makedirs(dst, exist_ok=True)
    for fn in os.listdir(src):
        if fn.endswith(".json") and fn != "model.safetensors.index.json" or fn.startswith("tokenizer") or fn.endswith(".model"):
            shutil.copy(os.path.join(src, fn), os.path.join(dst, fn))
    if qcfg is not None:
        p = os.path.join(dst, "config.json")
        cfg = json.load(open(p)) if os.path.exists(p) else {}
        cfg["quantization_config"] = qcfg
        json.dump(cfg, open(p, "w"), indent=2)


def _quantize_dir(src, dst, fn_quant, qcfg, device):
    _copy_meta(src, dst, qcfg)
    out, size, idx, wmap = {}, 0, 0, {}

    def flush():
        nonlocal out, size, idx
        if out:
            idx += 1
            name = f"model-{idx:05d}.safetensors"
            save_file(out, os.path.join(dst, name))
            wmap.update({k: name for k in out})
            out, size = {}, 0

    for _, k, t in _iter_hf(src):
        if _quantizable(k, t):
            for nk, nt in fn_quant(k, t.to(device)).items():
                out[nk] = nt.cpu().contiguous()
                size += nt.numel() * nt.element_size()
        else:
            out[k] = t
            size += t.numel() * t.element_size()
        if size > (4 << 30):
            flush()
    flush()
    json.dump({"metadata": {}, "weight_map": wmap}, open(os.path.join(dst, "model.safetensors.index.json"), "w"))


def hf2fp8(a):
    block = tuple(a.block)

    def q(k, t):
        w, s = Q.fp8_block_quant(t.to(torch.bfloat16), block, a.ue8m0)
        return {k: w, k + "_scale_inv": s}

    _quantize_dir(a.hf, a.out, q, {"quant_method": "fp8", "fmt": "e4m3", "activation_scheme": "dynamic",
                                   "weight_block_size": list(block)}, a.device)


def hf2int4(a):
    def q(k, t):
        if t.shape[1] % a.group:
            return {k: t}  # in-dim not a multiple of the group: keep bf16
        qq, s, z = Q.int4_fake_quant(t.to(torch.bfloat16), a.group, not a.asym)
        vals = (qq.float() + (0 if a.asym else 8)).to(torch.uint8)  # unsigned codes 0..15
        packed = vals[:, 0::2] | (vals[:, 1::2] << 4)
        d = {k.replace(".weight", ".weight_packed"): packed, k.replace(".weight", ".weight_scale"): s}
        if a.asym:
            d[k.replace(".weight", ".weight_zero_point")] = z
        return d

    _quantize_dir(a.hf, a.out, q, {"quant_method": "compressed-tensors", "format": "pack-quantized",
                                   "config_groups": {"group_0": {"weights": {
                                       "num_bits": 4, "group_size": a.group, "symmetric": not a.asym,
                                       "strategy": "group", "type": "int"}}}}, a.device)


def hf2nvfp4(a):
    def q(k, t):
        if t.shape[1] % 16:
            return {k: t}
        p, bs, gs = Q.nvfp4_quant(t.to(torch.bfloat16))
        return {k: p, k.replace(".weight", ".weight_scale"): bs,
                k.replace(".weight", ".weight_scale_2"): torch.tensor(gs, dtype=torch.float32)}

    _quantize_dir(a.hf, a.out, q, {"quant_method": "modelopt", "quant_algo": "NVFP4", "group_size": 16}, a.device)


def hf2mxfp8(a):
    def q(k, t):
        if t.shape[1] % 32:
            return {k: t}
        y, e = Q.mxfp8_quant(t.to(torch.bfloat16))
        return {k: y, k.replace(".weight", ".weight_scale"): e}

    _quantize_dir(a.hf, a.out, q, {"quant_method": "mxfp8", "group_size": 32}, a.device)


def fp8tobf16(a):
    tensors = {k: t for _, k, t in _iter_hf(a.hf)}
    out = {}
    for k, t in tensors.items():
        if k.endswith("_scale_inv"):
            continue
        s = tensors.get(k + "_scale_inv")
        out[k] = Q.fp8_block_dequant(t, s) if s is not None else t
    _copy_meta(a.hf, a.out)
    save_file(out, os.path.join(a.out, "model.safetensors"))


def hf2dist(a):
    from miles_b200.checkpoint.hf import load_hf
    from miles_b200.checkpoint.torch_dist import save_checkpoint
    from miles_b200.models.config import ModelConfig, preset
    from miles_b200.models.transformer import Transformer

    cfg = preset(a.model_name) if a.model_name else ModelConfig.from_hf(a.hf)
    m = Transformer(cfg, device=a.device, materialize=False)
    load_hf(m, a.hf)
    save_checkpoint(a.save, 0, m, None, save_optim=False)


def dist2hf(a):
    from miles_b200.checkpoint.hf import save_hf
    from miles_b200.checkpoint.torch_dist import load_checkpoint
    from miles_b200.models.config import ModelConfig, preset

    from miles_b200.models.transformer import Transformer

    cfg = preset(a.hf_config) if not os.path.exists(a.hf_config) else ModelConfig.from_hf(a.hf_config)
    m = Transformer(cfg, device=a.device, materialize=False)
    load_checkpoint(a.load, m, None, load_optim=False)
    save_hf(m, a.out)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("cmd", choices=["hf2dist", "dist2hf", "hf2fp8", "hf2int4", "hf2nvfp4", "hf2mxfp8", "fp8tobf16"])
    ap.add_argument("--hf")
    ap.add_argument("--out")
    ap.add_argument("--save")
    ap.add_argument("--load")
    ap.add_argument("--hf-config")
    ap.add_argument("--model-name")
    ap.add_argument("--block", type=int, nargs=2, default=[128, 128])
    ap.add_argument("--ue8m0", action="store_true")
    ap.add_argument("--group", type=int, default=128)
    ap.add_argument("--asym", action="store_true")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    globals()[a.cmd](a)


if __name__ == "__main__":
    main()
