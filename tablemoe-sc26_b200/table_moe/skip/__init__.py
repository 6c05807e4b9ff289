from .pruning import (
    build_decode_keep_mask,
    build_fixed_keep_mask,
    build_prefill_keep_mask,
    renormalize_surviving_weights,
)

__all__ = [
    "build_decode_keep_mask",
    "build_fixed_keep_mask",
    "build_prefill_keep_mask",
    "renormalize_surviving_weights",
]
