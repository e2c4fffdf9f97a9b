"""The gpt-oss entry points of the reference package, for training scripts written against it
(reference: src/agent_factory_3/models/gpt_oss/__init__.py, quantizer_config.py:49-61,
routing_replay.py:31-137).

There the model is a transformers ``GptOss`` model that needs a quantizer config (so that MXFP4
experts are dequantised on the fly) and a patch that threads recorded routes through the
decoder.  Here both are native to ``GptOssForCausalLM``: its experts stay MXFP4 and are
dequantised by this package's kernels, and ``forward_hidden`` takes ``routing_indices``.  The
names below keep such scripts working:

    cfg = Mxfp4Bf16DequantConfig(dequant_dtype="bf16")
    model = from_pretrained(MODEL_PATH, quantization_config=cfg, device="cuda")
    enable_routing_replay(model)
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from pathlib import Path

import torch

from .config import GptOssConfig, LoraConfig
from .model import GptOssForCausalLM

_DEQUANT_DTYPES = ("bf16", "fp8")


@dataclass
class Mxfp4Bf16DequantConfig:
    """How the frozen MXFP4 experts are computed on.

    ``dequant_dtype``: "bf16" dequantises to bf16 for the grouped expert GEMMs; "fp8" converts to
    e4m3 with one exact power-of-two scale per expert and runs the e4m3 tensor-core GEMM.
    ``fuse_swiglu`` is kept for the reference's config schema; the SwiGLU is always fused into
    the gate_up GEMM's epilogue here."""

    dequant_dtype: str = "bf16"
    fuse_swiglu: bool = True
    quant_method: str = "mxfp4_dequant"

    def __post_init__(self):
        if self.dequant_dtype not in _DEQUANT_DTYPES:
            raise ValueError(f"dequant_dtype must be one of {_DEQUANT_DTYPES}, "
                             f"got {self.dequant_dtype!r}")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict) -> "Mxfp4Bf16DequantConfig":
        return cls(**{k: d[k] for k in ("dequant_dtype", "fuse_swiglu", "quant_method") if k in d})

    def apply(self, model: GptOssForCausalLM) -> GptOssForCausalLM:
        for layer in model.layers:
            layer.mlp.dequant_dtype = self.dequant_dtype
        return model


def enable_routing_replay(model: GptOssForCausalLM) -> GptOssForCausalLM:
    """Routing replay is built into ``GptOssForCausalLM.forward_hidden(routing_indices=...)``
    ([T, L, K] expert ids; softmax over the K replayed logits, as the reference does), so there
    is nothing to patch.  Returns the model."""
    if not isinstance(model, GptOssForCausalLM):
        raise TypeError(f"expected GptOssForCausalLM, got {type(model).__name__}")
    return model


def from_pretrained(path: str | Path, quantization_config=None, device="cpu",
                    lora: LoraConfig | None = None, seed: int = 0,
                    dtype: torch.dtype = torch.bfloat16) -> GptOssForCausalLM:
    """Model from an HF gpt-oss checkpoint directory (config.json + MXFP4 safetensors) or a
    preset name (random weights).  ``quantization_config`` is a ``Mxfp4Bf16DequantConfig`` or
    its dict form; LoRA factors, if any, are initialised as PEFT does (B = 0)."""
    from .checkpoint import load_checkpoint
    p = Path(path)
    is_dir = p.is_dir() and (p / "config.json").exists()
    cfg = GptOssConfig.load(p / "config.json") if is_dir else GptOssConfig.preset(str(path))
    model = GptOssForCausalLM(cfg, lora=lora, device=device, dtype=dtype)
    if is_dir and any(p.glob("*.safetensors")):
        missing = load_checkpoint(p, model)
        if missing:
            raise RuntimeError(f"checkpoint {p} is missing {len(missing)} tensors, "
                               f"e.g. {missing[:3]}")
        if lora is not None:
            model.init_lora(seed=seed)
    else:
        model.init_random(seed=seed)
    qc = quantization_config
    if isinstance(qc, dict):
        qc = Mxfp4Bf16DequantConfig.from_dict(qc)
    (qc or Mxfp4Bf16DequantConfig()).apply(model)
    return model
