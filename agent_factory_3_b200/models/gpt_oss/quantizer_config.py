"""Module path of the reference's quantizer registration (models/gpt_oss/quantizer_config.py).
Nothing is registered here: the model is native and its MXFP4 experts are always dequantised
by this package's kernels; the config class selects the expert compute type."""
from .compat import Mxfp4Bf16DequantConfig

__all__ = ["Mxfp4Bf16DequantConfig"]
