"""Linear-algebra level functions of the framework: the functional attention
family (the reference keeps it in its linear-algebra crate)."""
from .attention import (  # noqa: F401
    AttentionConfig,
    AttentionMask,
    attention_with_alibi,
    attention_with_rpe,
    causal_attention,
    flash_attention,
    grouped_query_attention,
    linear_attention,
    masked_attention,
    multi_head_attention,
    relative_position_attention,
    rotary_embedding,
    scaled_dot_product_attention,
    sparse_attention,
)
