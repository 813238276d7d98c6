"""B200-native drop-in for MAGI-2's ``inference/flash_mh_moe``.

Same public names as the reference package (``inference/flash_mh_moe/__init__.py``):
``compute_topk_probs_and_indices``, ``flash_mh_moe_global_sort``, ``flash_mh_moe_fwd``.
All three run through libmhmoe (hand-written sm_100a CUDA behind a C ABI); the expert
FFN computes on NVFP4 operands with tcgen05 block-scaled tensor-core MMAs.
"""
from .fwd import flash_mh_moe_fwd
from .route import compute_topk_probs_and_indices, flash_mh_moe_global_sort

__all__ = [
    "compute_topk_probs_and_indices",
    "flash_mh_moe_global_sort",
    "flash_mh_moe_fwd",
]
