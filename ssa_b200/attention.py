"""Stage 3 of the ``ssa`` API: ``sparse_exact_attention`` and ``dense_attention``."""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from . import ops


def sparse_exact_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                           scale: Optional[float] = None, is_causal: bool = False,
                           q_offset: int = 0) -> torch.Tensor:
    """Exact softmax attention of each query over its selected keys
    (ssa/attention.py:12-115), on the sm_100a kernel.

    Args:
        q: ``[n, h_q, d]`` (or ``[B, n, h_q, d]``).
        k, v: ``[n, h_kv, d]`` (or ``[B, n, h_kv, d]``).
        indices: ``[n, h_kv, k]`` int64/int32 key positions per query and KV head.
        scale: logits are ``(q . k) / scale``; default ``sqrt(d)`` (a divisor,
            as in the reference).
        is_causal: mask keys ``j > q_offset + i``.  The reference applies no
            mask here; ``SSAAttention`` passes ``True`` so that filler keys of
            early queries never attend to the future.
        q_offset: sequence position of query row 0 (query-sharded calls).

    Keys are gathered per KV head (``k[idx, h]``), which corrects the
    reference's flattened gather for ``num_kv_heads > 1``.
    Returns a new ``[n, h_q, d]`` tensor in ``q``'s dtype.
    """
    unbatched = q.dim() == 3
    if unbatched:
        q, k, v, indices = q.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0), indices.unsqueeze(0)
    if q.shape[-2] % k.shape[-2]:
        raise ValueError("num_q_heads must be divisible by num_kv_heads")
    if scale is None:
        scale = math.sqrt(q.shape[-1])
    out = ops.sparse_attn(q, k, v, indices, float(scale), bool(is_causal), int(q_offset))
    return out[0] if unbatched else out


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    causal_mask: Optional[torch.Tensor] = None,
                    scale: Optional[float] = None) -> torch.Tensor:
    """Dense GQA softmax attention, the comparison path (ssa/attention.py:118-158).

    Plain PyTorch (``scaled_dot_product_attention``); ``scale`` divides the logits."""
    n, h_q, d = q.shape
    h_kv = k.shape[1]
    if scale is None:
        scale = math.sqrt(d)
    g = h_q // h_kv
    qt = q.transpose(0, 1).unsqueeze(0)
    kt = k.repeat_interleave(g, dim=1).transpose(0, 1).unsqueeze(0)
    vt = v.repeat_interleave(g, dim=1).transpose(0, 1).unsqueeze(0)
    mask = None if causal_mask is None else causal_mask.to(device=q.device, dtype=torch.bool)
    out = F.scaled_dot_product_attention(qt, kt, vt, attn_mask=mask, scale=1.0 / scale)
    return out[0].transpose(0, 1)
