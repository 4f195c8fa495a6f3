"""Module level of the ``ssa`` API: ``SSAAttention`` and ``ToyTransformerBlock``."""

from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn as nn

from .attention import dense_attention, sparse_exact_attention
from .router import CodebookRouter
from .utils import apply_rope, build_causal_mask

_README_ALIASES = {"d_model": "hidden_size", "h_q": "num_q_heads", "h_kv": "num_kv_heads",
                   "d_head": "head_dim", "d_s": "route_dim", "n_c": "num_codebook",
                   "b": "codes_per_key", "a": "codes_per_query", "k": "top_k"}


class SSAAttention(nn.Module):
    """Sub-quadratic selective attention layer (ssa/ssa_layer.py:17-138).

    Same constructor, parameters and state_dict keys as the reference
    (``q_proj``/``k_proj``/``v_proj``/``o_proj`` and ``router.*``); the README
    spelling ``SSAAttention(d_model=, h_q=, h_kv=, d_head=, d_s=, n_c=, b=, a=,
    k=, causal=)`` is accepted too.

    The reference loops over the batch in Python (ssa/ssa_layer.py:99); here
    the whole batch goes through one router launch sequence and one attention
    launch.  RoPE keeps the reference's convention (see :func:`apply_rope`).
    """

    def __init__(self, hidden_size: int = 512, num_q_heads: int = 8, num_kv_heads: int = 2,
                 head_dim: int = 64, route_dim: int = 16, num_codebook: int = 512,
                 codes_per_key: int = 4, codes_per_query: int = 8, top_k: int = 64,
                 bias: bool = False, causal: bool = True, **aliases):
        cfg = dict(hidden_size=hidden_size, num_q_heads=num_q_heads, num_kv_heads=num_kv_heads,
                   head_dim=head_dim, route_dim=route_dim, num_codebook=num_codebook,
                   codes_per_key=codes_per_key, codes_per_query=codes_per_query, top_k=top_k)
        for name, val in aliases.items():
            if name not in _README_ALIASES:
                raise TypeError(f"SSAAttention got an unexpected keyword argument '{name}'")
            cfg[_README_ALIASES[name]] = val
        super().__init__()
        if cfg["num_q_heads"] % cfg["num_kv_heads"]:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        self.hidden_size = cfg["hidden_size"]
        self.num_q_heads = cfg["num_q_heads"]
        self.num_kv_heads = cfg["num_kv_heads"]
        self.head_dim = cfg["head_dim"]
        self.top_k = cfg["top_k"]
        self.causal = causal
        hd = self.head_dim
        self.q_proj = nn.Linear(self.hidden_size, self.num_q_heads * hd, bias=bias)
        self.k_proj = nn.Linear(self.hidden_size, self.num_kv_heads * hd, bias=bias)
        self.v_proj = nn.Linear(self.hidden_size, self.num_kv_heads * hd, bias=bias)
        self.o_proj = nn.Linear(self.num_q_heads * hd, self.hidden_size, bias=bias)
        self.router = CodebookRouter(head_dim=hd, route_dim=cfg["route_dim"],
                                     num_kv_heads=self.num_kv_heads,
                                     num_codebook=cfg["num_codebook"],
                                     codes_per_key=cfg["codes_per_key"],
                                     codes_per_query=cfg["codes_per_query"], top_k=self.top_k)

    def _rope(self, x: torch.Tensor, freqs: torch.Tensor, position_ids: Optional[torch.Tensor]):
        # x: [B, n, h, d].  The reference rotates each batch element with
        # freqs_b = freqs[position_ids[b]] (or freqs[:n]) and apply_rope reads
        # rows 0..h-1 of freqs_b (ssa/ssa_layer.py:104-117, ssa/utils.py:19-24).
        n = x.shape[1]
        if position_ids is None:
            return apply_rope(x, freqs[:n])
        out = [apply_rope(x[b], freqs[position_ids[b]]) for b in range(x.shape[0])]
        return torch.stack(out, dim=0)

    def forward(self, hidden_states: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                position_ids: Optional[torch.Tensor] = None, freqs: Optional[torch.Tensor] = None,
                use_dense: bool = False) -> torch.Tensor:
        """``hidden_states [B, n, hidden]`` -> ``[B, n, hidden]``.

        ``attention_mask`` is accepted and ignored, as in the reference."""
        bsz, n, _ = hidden_states.shape
        hd = self.head_dim
        q = self.q_proj(hidden_states).view(bsz, n, self.num_q_heads, hd)
        k = self.k_proj(hidden_states).view(bsz, n, self.num_kv_heads, hd)
        v = self.v_proj(hidden_states).view(bsz, n, self.num_kv_heads, hd)
        if freqs is not None:
            q = self._rope(q, freqs, position_ids)
            k = self._rope(k, freqs, position_ids)
        if use_dense:
            mask = build_causal_mask(n, device=hidden_states.device) if self.causal else None
            out = torch.stack([dense_attention(q[b], k[b], v[b], causal_mask=mask) for b in range(bsz)])
        else:
            idx = self.router.route(q, k, causal=self.causal, index_dtype=torch.int32)[0]
            out = sparse_exact_attention(q, k, v, idx, scale=math.sqrt(hd), is_causal=self.causal)
        return self.o_proj(out.reshape(bsz, n, self.num_q_heads * hd))

    def compute_auxiliary_loss(self, hidden_states: torch.Tensor, freqs: Optional[torch.Tensor] = None):
        """The reference's training-time routing loss (KL divergence between
        the router's code scores and dense attention, ssa/ssa_layer.py:140-213)
        is not part of the forward hot path this package implements."""
        raise NotImplementedError("compute_auxiliary_loss is a router-training loss; ssa_b200 implements the "
                                  "forward path (routing + sparse attention) and its gradient")


class ToyTransformerBlock(nn.Module):
    """Pre-norm block: LayerNorm -> SSAAttention -> residual -> LayerNorm ->
    GELU MLP -> residual (ssa/ssa_layer.py:260-285)."""

    def __init__(self, hidden_size: int = 512, **ssa_kwargs):
        super().__init__()
        self.attn = SSAAttention(hidden_size=hidden_size, **ssa_kwargs)
        self.norm1 = nn.LayerNorm(hidden_size)
        self.norm2 = nn.LayerNorm(hidden_size)
        self.ffn = nn.Sequential(nn.Linear(hidden_size, 4 * hidden_size), nn.GELU(),
                                 nn.Linear(4 * hidden_size, hidden_size))

    def forward(self, x: torch.Tensor, **attn_kwargs) -> torch.Tensor:
        x = x + self.attn(self.norm1(x), **attn_kwargs)
        return x + self.ffn(self.norm2(x))
