"""gpt-oss (20b / 120b) with MXFP4 experts, LoRA and routing replay."""
from .config import GptOssConfig, LoraConfig
from .model import GptOssForCausalLM
from .compat import Mxfp4Bf16DequantConfig, enable_routing_replay, from_pretrained

__all__ = ["GptOssConfig", "LoraConfig", "GptOssForCausalLM", "Mxfp4Bf16DequantConfig",
           "enable_routing_replay", "from_pretrained"]
