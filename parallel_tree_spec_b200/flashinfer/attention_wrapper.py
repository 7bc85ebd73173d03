"""``parallel_tree_spec.flashinfer.attention_wrapper`` under its reference import path."""
from ..attention_wrapper import (  # noqa: F401
    FLASH_INFER_SUPPORTED_DIMS,
    POS_ENCODING_MODE,
    AttentionRotaryParams,
    BeFlashinferWrapper,
    find_padded_head_dim,
)
