"""Inference: paged KV cache, paged decode attention, speculative decoding,
and cached generation for the GPT engine."""
from .kv_cache import BlockManager, BlockManagerConfig, InferenceError, KvPageConfig, KvPagePool, SharedPrefixCache
from .paged_attention import PagedAttentionConfig, PagedAttentionForward, paged_attention_reference
from .generate import GPTGenerator
from .speculative import SpeculativeConfig, SpeculativeDecoder, SpeculativeResult, TokenDist, Xorshift64

__all__ = [
    "GPTGenerator",
    "BlockManager", "BlockManagerConfig", "InferenceError", "KvPageConfig", "KvPagePool", "SharedPrefixCache",
    "PagedAttentionConfig", "PagedAttentionForward", "paged_attention_reference",
    "SpeculativeConfig", "SpeculativeDecoder", "SpeculativeResult", "TokenDist", "Xorshift64",
]
