"""Stages 1-2 of the ``ssa`` API: ``CodebookRouter`` on the sm_100a kernels."""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops
from .utils import is_lower_triangular_mask

_README_ALIASES = {"d": "head_dim", "d_s": "route_dim", "n_c": "num_codebook", "b": "codes_per_key",
                   "a": "codes_per_query", "k": "top_k", "h_kv": "num_kv_heads"}


class CodebookRouter(nn.Module):
    """Content-dependent router: for every query position and KV head, the
    indices of ``top_k`` keys (ssa/router.py:14-275).

    Parameters and state_dict keys match the reference (``W_qr.weight``,
    ``W_kr.weight`` ``[route_dim, head_dim]``; ``codebook``
    ``[num_kv_heads, num_codebook, route_dim]``), so reference checkpoints
    load unchanged.  A shared ``[num_codebook, route_dim]`` codebook (the
    design-document form) is also accepted by :meth:`forward` via
    ``load_state_dict``/assignment and is broadcast to every head.

    The README spelling ``CodebookRouter(d=, d_s=, n_c=, b=, a=, k=)`` is
    accepted as well.
    """

    def __init__(self, head_dim: int = 128, route_dim: int = 32, num_kv_heads: int = 8,
                 num_codebook: int = 2048, codes_per_key: int = 4, codes_per_query: int = 16,
                 top_k: int = 256, temperature: float = 1.0, **aliases):
        cfg = dict(head_dim=head_dim, route_dim=route_dim, num_kv_heads=num_kv_heads,
                   num_codebook=num_codebook, codes_per_key=codes_per_key,
                   codes_per_query=codes_per_query, top_k=top_k)
        for name, val in aliases.items():
            if name not in _README_ALIASES:
                raise TypeError(f"CodebookRouter got an unexpected keyword argument '{name}'")
            cfg[_README_ALIASES[name]] = val
        super().__init__()
        self.head_dim = cfg["head_dim"]
        self.route_dim = cfg["route_dim"]
        self.num_kv_heads = cfg["num_kv_heads"]
        self.num_codebook = cfg["num_codebook"]
        self.codes_per_key = cfg["codes_per_key"]
        self.codes_per_query = cfg["codes_per_query"]
        self.top_k = cfg["top_k"]
        self.temperature = temperature
        self.W_qr = nn.Linear(self.head_dim, self.route_dim, bias=False)
        self.W_kr = nn.Linear(self.head_dim, self.route_dim, bias=False)
        self.codebook = nn.Parameter(
            torch.randn(self.num_kv_heads, self.num_codebook, self.route_dim) / self.route_dim ** 0.5)

    def _causal_flag(self, causal_mask: Optional[torch.Tensor], causal: Optional[bool]) -> bool:
        if causal is not None:
            return bool(causal)
        if causal_mask is None:
            return False
        if not is_lower_triangular_mask(causal_mask):
            raise ValueError("CodebookRouter supports no mask or the lower-triangular causal mask "
                             "(build_causal_mask); got another mask")
        return True

    def route(self, q_full: torch.Tensor, k_full: torch.Tensor, causal: bool = True,
              q_offset: int = 0, index_dtype: torch.dtype = torch.int64):
        """Batched routing: ``q [B, n_q, h_q, d]``, ``k [B, n, h_kv, d]`` ->
        ``(indices [B, n_q, h_kv, k], q_codes, k_codes, cand_counts)``."""
        if q_full.shape[-2] % k_full.shape[-2]:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        with torch.no_grad():
            return ops.route(q_full, k_full, self.W_qr.weight, self.W_kr.weight, self.codebook,
                             self.codes_per_query, self.codes_per_key, self.top_k, bool(causal),
                             float(self.temperature), int(q_offset), index_dtype == torch.int64)

    def route_rope(self, q_full: torch.Tensor, k_full: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                   causal: bool = True, q_offset: int = 0, index_dtype: torch.dtype = torch.int64):
        """RoPE + routing in one call, for the Qwen2 path of the reference
        (``training/train_qwen.py:134-135`` rotates with
        ``apply_rotary_pos_emb`` before the router): ``q [B, n_q, h_q, d]`` and
        ``k [B, n, h_kv, d]`` before RoPE, ``cos`` / ``sin`` the position
        tables (``[positions, d]``, ``[1|B, positions, d]`` or head-broadcast
        4-D forms, dtype of q/k).  The routing projection rotates each row as it
        loads it (``x * cos + rotate_half(x) * sin``, rounded as that PyTorch
        expression rounds) and writes the rotated rows out ->
        ``(indices [B, n_q, h_kv, k], q_rot, k_rot)``; attend with
        ``q_rot`` / ``k_rot``.  16-bit q/k, head_dim 64 or 128."""
        if q_full.shape[-2] % k_full.shape[-2]:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        with torch.no_grad():
            idx, _, _, _, q_rot, k_rot = ops.route_rope(
                q_full, k_full, cos, sin, self.W_qr.weight, self.W_kr.weight, self.codebook,
                self.codes_per_query, self.codes_per_key, self.top_k, bool(causal), float(self.temperature),
                int(q_offset), index_dtype == torch.int64)
        return idx, q_rot, k_rot

    def key_codes(self, k_full: torch.Tensor) -> torch.Tensor:
        """Batched key codes ``[B, n, h_kv, b]`` int32 of ``k [B, n, h_kv, d]``
        (the input :meth:`route_with_key_codes` takes)."""
        with torch.no_grad():
            return ops.code_assign(k_full, self.W_kr.weight, self.codebook, self.codes_per_key, 1.0)

    def route_with_key_codes(self, q_full: torch.Tensor, k_full: torch.Tensor, k_codes: torch.Tensor,
                             causal: bool = True, q_offset: int = 0,
                             index_dtype: torch.dtype = torch.int64) -> torch.Tensor:
        """:meth:`route` for the query rows ``q [B, n_q, h_q, d]`` at positions
        ``q_offset ..`` against all keys ``k [B, n, h_kv, d]`` whose codes are
        given (``k_codes [B, n, h_kv, b]``, e.g. gathered from per-shard
        :meth:`key_codes`) -> indices ``[B, n_q, h_kv, top_k]``."""
        if q_full.shape[-2] % k_full.shape[-2]:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        with torch.no_grad():
            return ops.route_with_key_codes(q_full, k_full, k_codes, self.W_qr.weight,
                                            self.W_kr.weight, self.codebook, self.codes_per_query,
                                            self.top_k, bool(causal), float(self.temperature),
                                            int(q_offset), index_dtype == torch.int64)

    def key_index(self, k_codes: torch.Tensor):
        """The code->key inverted index of ``k_codes [B, n, h_kv, b]``:
        ``(bucket_ptr [B, h_kv, N_c+1], bucket_keys [B, h_kv, n*b])``."""
        return ops.build_index(k_codes, self.num_codebook)

    def route_with_index(self, q_full: torch.Tensor, k_full: torch.Tensor, k_codes: torch.Tensor, index,
                         causal: bool = True, q_offset: int = 0,
                         index_dtype: torch.dtype = torch.int64) -> torch.Tensor:
        """:meth:`route_with_key_codes` with the index of ``k_codes`` given
        (``index`` from :meth:`key_index`), for several query blocks of one
        sequence against the same keys."""
        if q_full.shape[-2] % k_full.shape[-2]:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        with torch.no_grad():
            return ops.route_with_index(q_full, k_full, k_codes, index[0], index[1], self.W_qr.weight,
                                        self.W_kr.weight, self.codebook, self.codes_per_query, self.top_k,
                                        bool(causal), float(self.temperature), int(q_offset),
                                        index_dtype == torch.int64)

    def forward(self, q_full: torch.Tensor, k_full: torch.Tensor,
                causal_mask: Optional[torch.Tensor] = None, hard: bool = True,
                causal: Optional[bool] = None) -> torch.Tensor:
        """``q_full [n, h_q, d]``, ``k_full [n, h_kv, d]`` (RoPE applied) ->
        int64 indices ``[n, h_kv, top_k]`` (ssa/router.py:73-149).

        ``causal_mask`` may be ``None`` or the ``tril`` mask; ``causal=`` (the
        README form) overrides it.  ``hard=False`` (Gumbel assignment) is
        training-only and not provided.  Batched ``[B, n, h, d]`` inputs give
        ``[B, n, h_kv, top_k]``."""
        if not hard:
            raise NotImplementedError("hard=False (Gumbel-softmax code assignment) is training-only "
                                      "and is not part of the forward hot path")
        is_causal = self._causal_flag(causal_mask, causal)
        unbatched = q_full.dim() == 3
        q4 = q_full.unsqueeze(0) if unbatched else q_full
        k4 = k_full.unsqueeze(0) if unbatched else k_full
        idx = self.route(q4, k4, is_causal)[0]
        return idx[0] if unbatched else idx

    def get_code_assignment(self, k_full: torch.Tensor) -> torch.Tensor:
        """Top-``codes_per_key`` codes of each key ``[n, h_kv, b]`` (int64,
        ssa/router.py:261-275)."""
        unbatched = k_full.dim() == 3
        k4 = k_full.unsqueeze(0) if unbatched else k_full
        with torch.no_grad():
            codes = ops.code_assign(k4, self.W_kr.weight, self.codebook, self.codes_per_key, 1.0)
        codes = codes.long()
        return codes[0] if unbatched else codes
