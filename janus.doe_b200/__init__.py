"""B200-native decode engine for janus.DoE's token loop.

The own "living MoE" model (RoPE/GQA attention with the 30*tanh clamp, variable-k parliament
router over alive SwiGLU experts) and the `--host` GGUF path (packed Q8_0/Q4_K llama-family
model with a LoRA parliament after each FFN), decoded by hand-written sm_100a kernels behind
the C ABI in include/jdgpu.h.  This module is the Python binding of that ABI.
"""
from .jdgpu import *  # noqa: F401,F403
from .jdgpu import lib, exported_symbols, LIB_PATH  # noqa: F401

__version__ = "0.1.0"
