"""B200-native (sm_100a) causal multi-head attention for llm-gpu-5.

Import by name (the directory name is not an identifier):

    pkg = importlib.import_module("llm-gpu-5_b200")
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=768, num_heads=12,
                                                attention_precision="bf16"))

All compute runs in ``libattn_b200.so`` (C ABI: ``include/attn_b200.h``); importing fails if the
library has not been built.
"""
from ._lib import AttnError, DeviceWaitError, LIB_PATH, clear_device_error, launch_count, lib  # noqa: F401  (fails loudly if unbuilt)
from . import dp, graphs, mha_ops  # noqa: F401
from .mha import DeviceBuffer, GPTConfig, KVCache, MultiHeadAttention, Parameter  # noqa: F401
from .ffn import FeedForward  # noqa: F401
from .mha_ops import MHAController, get_shared_mha_module, THREADS_PER_BLOCK, SOFTMAX_BLOCK_THREADS  # noqa: F401

__all__ = ["MultiHeadAttention", "FeedForward", "GPTConfig", "Parameter", "DeviceBuffer", "KVCache", "mha_ops", "dp", "graphs", "AttnError", "DeviceWaitError", "clear_device_error",
           "get_shared_mha_module", "MHAController", "launch_count"]
