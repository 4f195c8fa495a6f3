"""ssa_b200 -- the SSA forward hot path on B200 (sm_100a).

A drop-in for the ``ssa`` package of chenxingqiang/SSA (``import ssa_b200 as
ssa``): the same public names (ssa/__init__.py:13-28), with the router
(stages 1-2) and sparse exact attention (stage 3) running as hand-written
CUDA kernels behind the C ABI in ``include/ssa_b200.h``.  CUDA tensors only.

Errors a kernel finds in the data (an index outside the sequence, a key code
outside the codebook) are raised without stalling the host: at a later op
call once the GPU has finished the failing one, or by :func:`check_errors`,
which waits for the GPU (``SSA_CHECKED=sync`` raises in the failing call).
"""

from ._status import check_errors
from .attention import dense_attention, sparse_exact_attention
from .layer import SSAAttention, ToyTransformerBlock
from .router import CodebookRouter
from .utils import (apply_rope, build_causal_mask, expand_kv_for_gqa, precompute_rope_freqs,
                    validate_indices)

__all__ = [
    "CodebookRouter",
    "sparse_exact_attention",
    "dense_attention",
    "SSAAttention",
    "ToyTransformerBlock",
    "apply_rope",
    "precompute_rope_freqs",
    "build_causal_mask",
    "expand_kv_for_gqa",
    "validate_indices",
]
