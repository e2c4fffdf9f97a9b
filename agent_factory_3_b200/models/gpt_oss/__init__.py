"""gpt-oss (20b / 120b) with MXFP4 experts, LoRA and routing replay."""
from .config import GptOssConfig, LoraConfig
from .model import GptOssForCausalLM

__all__ = ["GptOssConfig", "LoraConfig", "GptOssForCausalLM"]
