"""gpt-oss checkpoint I/O in the Hugging Face MXFP4 format, plus merged-weight export.

Key names are those of openai/gpt-oss checkpoints (``model.layers.{i}.self_attn.q_proj.weight``,
``model.layers.{i}.mlp.experts.gate_up_proj_blocks`` [E, 2I, H/32, 16] uint8,
``..._scales`` [E, 2I, H/32] uint8, ``..._bias``, ``model.layers.{i}.mlp.router.weight`` ...).
Sharded checkpoints (``model.safetensors.index.json``) are read shard by shard.

``merged_state_dict`` folds LoRA into the bf16 attention weights (W + s*B@A) and returns HF key
names, which is what the rollout engine loads on a merged-mode weight sync (reference:
trainer/model_trainer.py:653-721, which merges on rank 0's CPU in fp32).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from ...ops import mxfp4
from .config import GptOssConfig
from .model import GptOssForCausalLM


def _qkv_split(cfg: GptOssConfig):
    q, kv = cfg.q_size, cfg.kv_size
    return {"q_proj": (0, q), "k_proj": (q, q + kv), "v_proj": (q + kv, q + 2 * kv)}


def hf_state_dict(model: GptOssForCausalLM, include_experts: bool = True) -> dict:
    """Base weights under HF names (attention bf16, experts MXFP4, norms fp32->bf16)."""
    cfg = model.cfg
    sd = {"model.embed_tokens.weight": model.embed_tokens.detach(),
          "model.norm.weight": model.norm.detach().to(torch.bfloat16),
          "lm_head.weight": model.lm_head.detach()}
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        a, m = layer.self_attn, layer.mlp
        for name, (s, e) in _qkv_split(cfg).items():
            sd[p + f"self_attn.{name}.weight"] = a.qkv_weight[s:e].detach()
            sd[p + f"self_attn.{name}.bias"] = a.qkv_bias[s:e].detach().to(torch.bfloat16)
        sd[p + "self_attn.o_proj.weight"] = a.o_weight.detach()
        sd[p + "self_attn.o_proj.bias"] = a.o_bias.detach().to(torch.bfloat16)
        sd[p + "self_attn.sinks"] = a.sinks.detach().to(torch.bfloat16)
        sd[p + "input_layernorm.weight"] = layer.input_layernorm.detach().to(torch.bfloat16)
        sd[p + "post_attention_layernorm.weight"] = layer.post_attention_layernorm.detach().to(torch.bfloat16)
        sd[p + "mlp.router.weight"] = m.router_weight.detach()
        sd[p + "mlp.router.bias"] = m.router_bias.detach().to(torch.bfloat16)
        if include_experts:
            sh = getattr(m, "expert_shards", None)     # sharded base: gather every rank's experts
            full = (lambda key, t: sh.packed(key, t)) if sh is not None else (lambda key, t: t)
            sd[p + "mlp.experts.gate_up_proj_blocks"] = full("gu_blocks", m.gate_up_blocks)
            sd[p + "mlp.experts.gate_up_proj_scales"] = full("gu_scales", m.gate_up_scales)
            sd[p + "mlp.experts.down_proj_blocks"] = full("dn_blocks", m.down_blocks)
            sd[p + "mlp.experts.down_proj_scales"] = full("dn_scales", m.down_scales)
        sd[p + "mlp.experts.gate_up_proj_bias"] = m.gate_up_bias.detach().to(torch.bfloat16)
        sd[p + "mlp.experts.down_proj_bias"] = m.down_bias.detach().to(torch.bfloat16)
    return sd


@torch.no_grad()
def load_state_dict_into(model: GptOssForCausalLM, get) -> list[str]:
    """Copy weights from ``get(name) -> tensor | None`` into ``model``; returns missing keys."""
    cfg = model.cfg
    missing = []

    def cp(dst, name, transform=None):
        t = get(name)
        if t is None:
            missing.append(name)
            return
        if transform is not None:
            t = transform(t)
        dst.copy_(t.to(device=dst.device, dtype=dst.dtype))

    cp(model.embed_tokens, "model.embed_tokens.weight")
    cp(model.norm, "model.norm.weight")
    cp(model.lm_head, "lm_head.weight")
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        a, m = layer.self_attn, layer.mlp
        for name, (s, e) in _qkv_split(cfg).items():
            cp(a.qkv_weight[s:e], p + f"self_attn.{name}.weight")
            cp(a.qkv_bias[s:e], p + f"self_attn.{name}.bias")
        cp(a.o_weight, p + "self_attn.o_proj.weight")
        cp(a.o_bias, p + "self_attn.o_proj.bias")
        cp(a.sinks, p + "self_attn.sinks")
        cp(layer.input_layernorm, p + "input_layernorm.weight")
        cp(layer.post_attention_layernorm, p + "post_attention_layernorm.weight")
        cp(m.router_weight, p + "mlp.router.weight")
        cp(m.router_bias, p + "mlp.router.bias")
        cp(m.gate_up_bias, p + "mlp.experts.gate_up_proj_bias")
        cp(m.down_bias, p + "mlp.experts.down_proj_bias")
        if get(p + "mlp.experts.gate_up_proj_blocks") is not None:
            cp(m.gate_up_blocks, p + "mlp.experts.gate_up_proj_blocks")
            cp(m.gate_up_scales, p + "mlp.experts.gate_up_proj_scales")
            cp(m.down_blocks, p + "mlp.experts.down_proj_blocks")
            cp(m.down_scales, p + "mlp.experts.down_proj_scales")
        else:  # bf16 experts in HF orientation [E, in, out] -> quantize
            gu = get(p + "mlp.experts.gate_up_proj")
            dn = get(p + "mlp.experts.down_proj")
            if gu is None or dn is None:
                missing.append(p + "mlp.experts.*")
                continue
            b, s = mxfp4.quantize(gu.transpose(1, 2).float())
            m.gate_up_blocks.copy_(b.to(m.gate_up_blocks.device))
            m.gate_up_scales.copy_(s.to(m.gate_up_scales.device))
            b, s = mxfp4.quantize(dn.transpose(1, 2).float())
            m.down_blocks.copy_(b.to(m.down_blocks.device))
            m.down_scales.copy_(s.to(m.down_scales.device))
    return missing


def load_checkpoint(path: str | Path, model: GptOssForCausalLM) -> list[str]:
    """Load an HF-format gpt-oss checkpoint directory (single file or sharded)."""
    path = Path(path)
    index = path / "model.safetensors.index.json"
    if index.exists():
        weight_map = json.loads(index.read_text())["weight_map"]
        files = sorted(set(weight_map.values()))
    else:
        files = [f.name for f in path.glob("*.safetensors")]
        weight_map = None
    handles = {f: safe_open(str(path / f), framework="pt") for f in files}
    keys = {}
    for f, h in handles.items():
        for k in h.keys():
            keys[k] = f

    def get(name):
        f = keys.get(name)
        return None if f is None else handles[f].get_tensor(name)

    return load_state_dict_into(model, get)


def save_checkpoint(model: GptOssForCausalLM, path: str | Path, shard_bytes: int = 5 << 30):
    """Write config.json and (sharded) model safetensors in the HF MXFP4 layout."""
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    cfg = model.cfg.to_hf_dict()
    cfg["quantization_config"] = {"quant_method": "mxfp4",
                                  "modules_to_not_convert": ["model.layers.*.self_attn",
                                                             "model.layers.*.mlp.router",
                                                             "model.embed_tokens", "lm_head"]}
    (path / "config.json").write_text(json.dumps(cfg, indent=2))
    sd = {k: v.detach().contiguous().cpu() for k, v in hf_state_dict(model).items()}
    shards, cur, size = [], {}, 0
    for k, v in sd.items():
        nb = v.numel() * v.element_size()
        if cur and size + nb > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = v
        size += nb
    shards.append(cur)
    if len(shards) == 1:
        save_file(shards[0], str(path / "model.safetensors"), metadata={"format": "pt"})
        return
    weight_map = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, str(path / fn), metadata={"format": "pt"})
        weight_map.update({k: fn for k in sh})
    (path / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {"total_size": sum(v.numel() * v.element_size() for v in sd.values())},
                    "weight_map": weight_map}, indent=2))


@torch.no_grad()
def merged_state_dict(model: GptOssForCausalLM, dtype=torch.bfloat16,
                      attention_only: bool = True) -> dict:
    """HF-named weights with LoRA folded in: W' = W + s * B @ A (fp32 math on the device).

    With ``attention_only`` (the default, as the reference's merged sync) only the attention
    projections are emitted; otherwise expert LoRA is folded into dequantised experts too and
    the experts are re-emitted in bf16 ``gate_up_proj`` / ``down_proj`` HF orientation."""
    cfg = model.cfg
    out = {}
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        a, m = layer.self_attn, layer.mlp
        s = a.lora_scaling
        for name, (lo, hi) in _qkv_split(cfg).items():
            w = a.qkv_weight[lo:hi].float()
            if f"{name}_A" in a.lora:
                w = w + s * (a.lora[f"{name}_B"].float() @ a.lora[f"{name}_A"].float())
            out[p + f"self_attn.{name}.weight"] = w.to(dtype)
        w = a.o_weight.float()
        if "o_proj_A" in a.lora:
            w = w + s * (a.lora["o_proj_B"].float() @ a.lora["o_proj_A"].float())
        out[p + "self_attn.o_proj.weight"] = w.to(dtype)
        if not attention_only:
            ex = m.experts()        # gathers the stacks when the base is sharded
            gu = ex.gate_up().float()
            dn = ex.down().float()
            if "gu_A" in m.lora:
                gu = gu + m.lora_scaling * torch.bmm(m.lora["gu_B"].float(), m.lora["gu_A"].float())
            if "dn_A" in m.lora:
                dn = dn + m.lora_scaling * torch.bmm(m.lora["dn_B"].float(), m.lora["dn_A"].float())
            out[p + "mlp.experts.gate_up_proj"] = gu.transpose(1, 2).contiguous().to(dtype)
            out[p + "mlp.experts.down_proj"] = dn.transpose(1, 2).contiguous().to(dtype)
    return out
