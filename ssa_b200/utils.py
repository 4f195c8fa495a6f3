"""Torch helpers of the ``ssa`` API: RoPE, causal masks, GQA expansion.

These stay plain PyTorch (they are glue around the hot path).  Semantics
follow the reference helpers in ssa/utils.py.
"""

from __future__ import annotations

import torch


def precompute_rope_freqs(head_dim: int, seq_len: int, theta: float = 10000.0, device=None) -> torch.Tensor:
    """RoPE angles ``[seq_len, head_dim // 2]`` (ssa/utils.py:51-72).

    ``dim = head_dim // 2`` features rotate; pair ``t`` of the ``dim // 2``
    pairs turns at ``theta ** (-2t / dim)`` rad per position; the angle table
    is repeated twice along the last axis (cos/sin halves)."""
    dim = head_dim // 2
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device).float() / dim))
    pos = torch.arange(seq_len, device=device, dtype=torch.float32)
    ang = pos[:, None] * inv[None, :]
    return torch.cat((ang, ang), dim=-1)


def apply_rope(x: torch.Tensor, freqs: torch.Tensor) -> torch.Tensor:
    """Rotary embedding with the reference's conventions (ssa/utils.py:7-48).

    The second-to-last axis of ``x`` indexes the rows of ``freqs``; only the
    first ``head_dim // 2`` features rotate (pairs ``(t, t + head_dim // 4)``),
    the rest pass through.  On the ``[seq, heads, d]`` tensors the reference's
    ``SSAAttention`` passes in, this rotates by head index -- reproduced here
    unchanged for module-level parity."""
    rows, d = x.shape[-2], x.shape[-1]
    half = d // 2
    quarter = half // 2
    ct = torch.promote_types(x.dtype, torch.float32)      # compute in >= fp32
    ang = freqs[:rows, :half].to(ct)
    cos, sin = ang.cos(), ang.sin()
    xf = x.to(ct)
    lo, hi = xf[..., :quarter], xf[..., quarter:half]
    c_lo, c_hi = cos[..., :quarter], cos[..., quarter:half]
    s_lo, s_hi = sin[..., :quarter], sin[..., quarter:half]
    rot = torch.cat((lo * c_lo - hi * s_lo, hi * c_hi + lo * s_hi), dim=-1).to(x.dtype)
    return torch.cat((rot, x[..., half:]), dim=-1)


def build_causal_mask(seq_len: int, device=None) -> torch.Tensor:
    """``[seq_len, seq_len]`` bool mask, True where ``j <= i`` (ssa/utils.py:75-86)."""
    m = torch.ones(seq_len, seq_len, dtype=torch.bool, device=device).tril_()
    m._ssa_lower_triangular = True
    return m


def is_lower_triangular_mask(mask: torch.Tensor) -> bool:
    """True if ``mask`` is exactly the ``tril`` causal mask."""
    if getattr(mask, "_ssa_lower_triangular", False):
        return True
    if mask.dim() != 2 or mask.shape[0] != mask.shape[1] or mask.dtype != torch.bool:
        return False
    n = mask.shape[0]
    return bool(torch.equal(mask, torch.ones(n, n, dtype=torch.bool, device=mask.device).tril_()))


def expand_kv_for_gqa(kv: torch.Tensor, num_q_heads: int, num_kv_heads: int) -> torch.Tensor:
    """``[..., h_kv, d]`` -> ``[..., h_q, d]`` exactly as the reference helper
    returns it (ssa/utils.py:89-106): the whole run of KV heads is tiled
    ``num_q_heads // num_kv_heads`` times, so query head ``j`` gets KV head
    ``j % num_kv_heads``.

    Note that this is not the pairing the attention itself uses: the router,
    ``sparse_exact_attention`` and ``dense_attention`` (here and in the
    reference, ssa/router.py:108-112, ssa/attention.py:143-146) give query head
    ``j`` KV head ``j // (num_q_heads // num_kv_heads)``.  The helper keeps the
    reference's output because it is part of the public API; nothing on the
    hot path calls it."""
    if num_q_heads % num_kv_heads:
        raise ValueError("num_q_heads must be divisible by num_kv_heads")
    g = num_q_heads // num_kv_heads
    tiled = kv.unsqueeze(-3).expand(*kv.shape[:-2], g, kv.shape[-2], kv.shape[-1])
    return tiled.reshape(*kv.shape[:-2], num_q_heads, kv.shape[-1])


def validate_indices(indices: torch.Tensor, seq_len: int, max_k: int, name: str = "indices") -> None:
    """Shape and range checks of candidate indices (ssa/utils.py:109-120)."""
    if indices.dim() < 2:
        raise ValueError(f"{name} must have at least 2 dims, got shape {tuple(indices.shape)}")
    if indices.shape[-1] > max_k:
        raise ValueError(f"{name} last dim {indices.shape[-1]} exceeds max_k {max_k}")
    if indices.numel() and (int(indices.max()) >= seq_len or int(indices.min()) < 0):
        raise ValueError(f"{name} has values outside [0, {seq_len})")
