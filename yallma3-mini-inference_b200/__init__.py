"""yallma3_b200 — B200-native (sm_100a) quantized-weight LLaMA forward path.

A drop-in for the hot path of yallma3-mini-inference: the Transformer trait,
the WeightType quantize/matmul entry points, the Q8_0 activation quantizer,
the GGUF loader and load_transformer_ffi, all behind the C-ABI in
include/yallma3.h and implemented by hand-written CUDA kernels
(libyallma3_b200.so, built in-tree by build.py).

The directory name contains hyphens; import it with
`importlib.import_module("yallma3-mini-inference_b200")` after putting the
repository root on sys.path (see load_package()).
"""
from .api import *  # noqa: F401,F403
from .api import (EXPORTED, LIB_PATH, PRESETS, InferenceSession, QuantizedTensor, Transformer, WeightFormat,
                  YlError, load_transformer, load_transformer_ffi, matmul, new_workspace_buffer, quantize,
                  quantize_q8_0, raw_lib, synth_preset, synth_write_gguf)
