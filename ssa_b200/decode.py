"""Token-by-token SSA decoding over a growing key/value cache.

Each step appends the new position's key and value, assigns the key its
codes once (``ssa_code_assign`` on that row only), routes the new query
against every cached key with the cached codes (``ssa_route_with_key_codes``,
``q_offset`` = the query's position) and attends over the selected keys
(``ssa_sparse_attn``).  A key's codes depend on that key alone, so the cache
holds each key's codes from the step it arrived in; the code->key index of
the cache is rebuilt inside the routing call (one pass over ``n * b`` codes).

The reference has no decode path (its design notes it, ``ssa_design.md``);
a step computes what ``CodebookRouter.forward`` + ``sparse_exact_attention``
compute for the last row of the sequence so far (``ssa/router.py:73-149``,
``ssa/attention.py:12-115``).  While fewer than ``top_k`` keys are cached the
indices are zero-padded as the reference pads ``k > n``
(``ssa/router.py:206-211``), so from position ``top_k - 1`` on a step equals
the full-sequence forward's row.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import ops


class DecodeCache:
    """Keys, values and key codes of ``batch`` sequences, up to ``capacity``
    positions each, on one GPU."""

    def __init__(self, router, batch: int, capacity: int, num_q_heads: int, dtype=torch.bfloat16,
                 device="cuda"):
        self.router = router
        self.batch, self.capacity = batch, capacity
        self.h_q, self.h_kv, self.d = num_q_heads, router.num_kv_heads, router.head_dim
        if self.h_q % self.h_kv:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        shape = (batch, capacity, self.h_kv, self.d)
        self.k = torch.empty(shape, dtype=dtype, device=device)
        self.v = torch.empty(shape, dtype=dtype, device=device)
        self.codes = torch.empty((batch, capacity, self.h_kv, router.codes_per_key), dtype=torch.int32,
                                 device=device)
        self.n = 0

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Adds ``t`` positions: ``k_new``, ``v_new`` ``[batch, t, h_kv, d]``."""
        t = k_new.shape[1]
        if self.n + t > self.capacity:
            raise ValueError(f"cache full: {self.n} + {t} > {self.capacity}")
        s = slice(self.n, self.n + t)
        self.k[:, s] = k_new
        self.v[:, s] = v_new
        self.codes[:, s] = self.router.key_codes(self.k[:, s])
        self.n += t

    def step(self, q_new: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             scale: Optional[float] = None) -> torch.Tensor:
        """One decoding step: appends position ``n`` (``k_new``, ``v_new``
        ``[batch, 1, h_kv, d]``) and returns the attention output of its query
        ``q_new [batch, 1, h_q, d]`` over the routed keys, ``[batch, 1, h_q, d]``."""
        self.append(k_new, v_new)
        n = self.n
        k, v = self.k[:, :n], self.v[:, :n]
        codes = self.codes[:, :n]
        idx = self.router.route_with_key_codes(q_new, k, codes, causal=True, q_offset=n - 1,
                                               index_dtype=torch.int32)
        if scale is None:
            scale = math.sqrt(self.d)
        return ops.sparse_attn(q_new, k, v, idx, float(scale), True, n - 1)
