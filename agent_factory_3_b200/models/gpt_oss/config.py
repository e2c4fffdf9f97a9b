"""gpt-oss architecture and LoRA configuration.

Field names follow the Hugging Face ``config.json`` of openai/gpt-oss-{20b,120b} so
checkpoints round-trip; presets cover the two released sizes and the tiny CPU-oracle
configuration used by the tests.
"""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path

GPT_OSS_ROPE_SCALING = {
    "rope_type": "yarn",
    "factor": 32.0,
    "beta_fast": 32.0,
    "beta_slow": 1.0,
    "truncate": False,
    "original_max_position_embeddings": 4096,
}


def _alternating_layer_types(n: int) -> list[str]:
    return ["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(n)]


@dataclass
class GptOssConfig:
    vocab_size: int = 201088
    hidden_size: int = 2880
    intermediate_size: int = 2880
    num_hidden_layers: int = 36
    num_attention_heads: int = 64
    num_key_value_heads: int = 8
    head_dim: int = 64
    num_local_experts: int = 128
    num_experts_per_tok: int = 4
    sliding_window: int = 128
    layer_types: list[str] = field(default_factory=list)
    rope_theta: float = 150000.0
    rope_scaling: dict | None = field(default_factory=lambda: dict(GPT_OSS_ROPE_SCALING))
    max_position_embeddings: int = 131072
    rms_norm_eps: float = 1e-5
    swiglu_limit: float = 7.0
    swiglu_alpha: float = 1.702
    attention_bias: bool = True
    initializer_range: float = 0.02
    eos_token_id: int = 200002
    pad_token_id: int = 199999
    tie_word_embeddings: bool = False

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = _alternating_layer_types(self.num_hidden_layers)
        assert len(self.layer_types) == self.num_hidden_layers
        assert self.hidden_size % 32 == 0 and self.intermediate_size % 32 == 0
        for name in ("pad_token_id", "eos_token_id"):
            v = getattr(self, name)
            if not 0 <= v < self.vocab_size:
                raise ValueError(f"{name}={v} is outside the vocabulary (size {self.vocab_size})")

    # ---- derived sizes ----
    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    def window(self, layer: int) -> int:
        return self.sliding_window if self.layer_types[layer] == "sliding_attention" else 0

    # ---- (de)serialisation ----
    def to_hf_dict(self) -> dict:
        d = asdict(self)
        d["model_type"] = "gpt_oss"
        d["architectures"] = ["GptOssForCausalLM"]
        d["experts_per_token"] = self.num_experts_per_tok
        d["num_experts"] = self.num_local_experts
        return d

    @classmethod
    def from_hf_dict(cls, d: dict) -> "GptOssConfig":
        known = {f for f in cls.__dataclass_fields__}
        kw = {k: v for k, v in d.items() if k in known}
        if "rope_parameters" in d and "rope_scaling" not in d:
            rp = dict(d["rope_parameters"])
            kw["rope_theta"] = rp.pop("rope_theta", kw.get("rope_theta", 150000.0))
            kw["rope_scaling"] = rp if rp.get("rope_type", "default") != "default" else None
        return cls(**kw)

    def save(self, path: str | Path) -> None:
        Path(path).write_text(json.dumps(self.to_hf_dict(), indent=2))

    @classmethod
    def load(cls, path: str | Path) -> "GptOssConfig":
        return cls.from_hf_dict(json.loads(Path(path).read_text()))

    # ---- presets ----
    @classmethod
    def gpt_oss_120b(cls) -> "GptOssConfig":
        return cls(num_hidden_layers=36, num_local_experts=128)

    @classmethod
    def gpt_oss_20b(cls) -> "GptOssConfig":
        return cls(num_hidden_layers=24, num_local_experts=32)

    @classmethod
    def tiny(cls) -> "GptOssConfig":
        """The CPU fp32 oracle configuration: 2 layers, hidden 64, 4 q / 2 kv heads of 16,
        alternating sliding-16 / full attention with sinks, 4 experts top-2, vocab 1024,
        RoPE theta 150000 (no YaRN)."""
        return cls(vocab_size=1024, hidden_size=64, intermediate_size=64, num_hidden_layers=2,
                   num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                   num_local_experts=4, num_experts_per_tok=2, sliding_window=16,
                   rope_scaling=None, max_position_embeddings=4096, eos_token_id=1,
                   pad_token_id=0)

    @classmethod
    def preset(cls, name: str) -> "GptOssConfig":
        return {"gpt-oss-120b": cls.gpt_oss_120b, "gpt-oss-20b": cls.gpt_oss_20b,
                "tiny": cls.tiny}[name]()


ATTN_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj")
EXPERT_TARGETS = ("gate_up_proj", "down_proj")


@dataclass
class LoraConfig:
    """LoRA adapter settings; ``target_modules`` uses PEFT names.  ``gate_up_proj`` /
    ``down_proj`` target the MoE experts (one rank-r factor pair per expert)."""

    r: int = 8
    lora_alpha: float = 32.0
    target_modules: list[str] = field(default_factory=lambda: list(ATTN_TARGETS))
    lora_dropout: float = 0.0

    @property
    def scaling(self) -> float:
        return self.lora_alpha / self.r

    def targets(self, name: str) -> bool:
        return name in self.target_modules

    def to_peft_dict(self, base_model: str = "") -> dict:
        attn = [t for t in self.target_modules if t in ATTN_TARGETS]
        experts = [f"mlp.experts.{t}" for t in self.target_modules if t in EXPERT_TARGETS]
        return {
            "peft_type": "LORA",
            "task_type": "CAUSAL_LM",
            "base_model_name_or_path": base_model,
            "r": self.r,
            "lora_alpha": self.lora_alpha,
            "lora_dropout": self.lora_dropout,
            "target_modules": attn,
            "target_parameters": experts or None,
            "bias": "none",
            "fan_in_fan_out": False,
            "inference_mode": True,
            "use_rslora": False,
            "use_dora": False,
        }

    @classmethod
    def from_peft_dict(cls, d: dict) -> "LoraConfig":
        targets = list(d.get("target_modules") or [])
        for t in d.get("target_parameters") or []:
            targets.append(t.split(".")[-1])
        return cls(r=int(d["r"]), lora_alpha=float(d["lora_alpha"]), target_modules=targets,
                   lora_dropout=float(d.get("lora_dropout", 0.0)))
