"""Torch-CPU port of the reference forward, timed as the CPU baseline --
BENCHMARK INFRASTRUCTURE ONLY.

Only ``bench.py`` (its ``cpu_baseline`` leg and its ``--impl reference`` arm)
and the tests that check this module may import it; the shipped path never
does.

The reference (chenxingqiang/SSA) is pure Python over PyTorch with no
packaging, so it is not installed on the GPU box.  This module restates its
forward with the same kinds of torch CPU operations, so that the timed CPU
baseline costs about what the reference's own code costs:

* the projection of every query head, then the GQA group mean
  (``ssa/router.py:102-112``);
* cosine scores against the normalised codebook by ``einsum`` and
  ``torch.topk`` for the a query / b key codes (``ssa/router.py:116-141``);
* the dense full-dimension re-score of every (query, key) pair with the
  group-mean logit, causal ``-inf`` and candidate ``-inf``, then
  ``topk(min(k, n))`` with zero padding (``ssa/router.py:151-214``).  The
  candidate mask uses a per-query code-membership table instead of the
  reference's broadcast comparison of all code pairs
  (``ssa/router.py:216-259``), which is a cheaper way to the same mask; the
  re-score runs per KV head and per block of query rows (the reference
  materialises it all at once and runs out of memory above n ~ 8K);
* the materialised gather of the selected K and V rows and ``einsum``
  attention (``ssa/attention.py:93-113``), with the per-head gather
  ``k[idx, h]`` and the causal mask.

Ties are broken by ``torch.topk``, as in the reference, not by the oracle's
stable rule; ``tests/test_oracle_golden.py`` checks this port against the
numpy oracle (``ssa_oracle``) on tie-free inputs.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def key_codes(k_h: torch.Tensor, w_kr: torch.Tensor, cb_h: torch.Tensor, b: int) -> torch.Tensor:
    """Top-b codes of the keys of one KV head: ``k_h [n, d]`` -> ``[n, b]``."""
    k_route = F.normalize(k_h @ w_kr.t(), dim=-1)
    scores = torch.einsum("nd,cd->nc", k_route, F.normalize(cb_h, dim=-1))
    return scores.topk(b, dim=-1).indices


def query_codes(q_h: torch.Tensor, w_qr: torch.Tensor, cb_h: torch.Tensor, a: int) -> torch.Tensor:
    """Top-a codes of the query rows of one KV head: ``q_h [rows, g, d]`` -> ``[rows, a]``."""
    q_route = F.normalize((q_h @ w_qr.t()).mean(dim=1), dim=-1)
    scores = torch.einsum("nd,cd->nc", q_route, F.normalize(cb_h, dim=-1))
    return scores.topk(a, dim=-1).indices


def select(q_h: torch.Tensor, k_h: torch.Tensor, q_codes: torch.Tensor, k_codes: torch.Tensor, n_codes: int,
           top_k: int, q_start: int = 0, causal: bool = True, block: int = 128) -> torch.Tensor:
    """Dense re-score + candidate mask + top-k for query rows at positions
    ``q_start ..`` of one KV head -> indices ``[rows, top_k]`` (int64)."""
    rows, g, d = q_h.shape
    n = k_h.shape[0]
    eff = min(top_k, n)
    out = torch.zeros((rows, top_k), dtype=torch.int64)
    jj = torch.arange(n)
    inv = 1.0 / math.sqrt(d)
    for i0 in range(0, rows, block):
        i1 = min(i0 + block, rows)
        logits = torch.einsum("rgd,nd->rgn", q_h[i0:i1], k_h) * inv
        sc = logits.mean(dim=1)                                           # [blk, n]
        if causal:
            pos = torch.arange(q_start + i0, q_start + i1)
            sc = sc.masked_fill(jj[None, :] > pos[:, None], float("-inf"))
        member = torch.zeros((i1 - i0, n_codes), dtype=torch.bool)
        member.scatter_(1, q_codes[i0:i1], True)
        cand = member[:, k_codes.reshape(-1)].reshape(i1 - i0, n, -1).any(dim=-1)
        sc = sc.masked_fill(~cand, float("-inf"))
        out[i0:i1, :eff] = sc.topk(eff, dim=-1).indices
    return out


def attention(q_h: torch.Tensor, k_h: torch.Tensor, v_h: torch.Tensor, idx: torch.Tensor, q_start: int = 0,
              causal: bool = True, block: int = 512) -> torch.Tensor:
    """Sparse exact attention of query rows at positions ``q_start ..`` over
    their selected keys (one KV head): ``[rows, g, d]``."""
    rows, g, d = q_h.shape
    out = torch.empty_like(q_h)
    inv = 1.0 / math.sqrt(d)
    for i0 in range(0, rows, block):
        i1 = min(i0 + block, rows)
        ib = idx[i0:i1]
        k_sel = k_h[ib]                                                   # [blk, kk, d]
        v_sel = v_h[ib]
        logits = torch.einsum("rgd,rkd->rgk", q_h[i0:i1], k_sel) * inv
        if causal:
            pos = torch.arange(q_start + i0, q_start + i1)
            logits = logits.masked_fill((ib > pos[:, None])[:, None, :], float("-inf"))
        p = torch.softmax(logits, dim=-1)
        out[i0:i1] = torch.einsum("rgk,rkd->rgd", p, v_sel)
    return out
