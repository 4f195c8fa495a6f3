"""CPU oracle for the SSA forward hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and its
``--impl reference`` arm) may import it.  The shipped path
(``ssa_b200`` + ``libssa_sm100a.so``) never calls into it and has no CPU
fallback.

It restates, in numpy, the reference implementation of chenxingqiang/SSA:

* stage 1 (routing projection, cosine codebook scores, top-b / top-a codes)
  -- ``ssa/router.py:102-141`` and ``ssa/router.py:261-275``;
* stage 2 (candidate mask, full-dimension group-mean re-score, causal mask,
  top-k with zero padding) -- ``ssa/router.py:151-259``;
* stage 3 (sparse exact attention) -- ``ssa/attention.py:12-115``;
* dense attention -- ``ssa/attention.py:118-158``.

Three documented corrections turn the reference into a well-defined oracle
(the reference leaves these implementation-defined or gets them wrong):

1. Every top-k is *stable*: among equal scores the lower index wins
   (``torch.topk`` tie order is unspecified, ``ssa/router.py:130,141,204``).
2. When a query has fewer than ``min(k, n)`` candidates the reference's
   ``topk`` returns arbitrary ``-inf`` entries (``ssa/router.py:200-204``);
   here the filler is the lowest-index non-candidate keys, in index order.
3. Stage 3 gathers ``k[idx, h]`` per KV head.  The reference's flattened
   gather offsets by ``h * seq_len`` into a ``[seq*h_kv, d]`` view
   (``ssa/attention.py:76-91``), which picks wrong rows whenever
   ``num_kv_heads > 1``.  With ``causal=True`` stage 3 also masks keys
   ``j > i`` (the reference applies no mask in stage 3), so filler never
   attends to the future and ``k = n`` reproduces dense causal attention.

Parity of this restatement is pinned against the reference itself, run in
the build container, through the committed fixtures in ``tests/golden/``
(made by ``tests/golden/make_golden.py``): stage-1 codes, the candidate mask,
top-k rows whose selection is well defined, stage 3 at ``h_kv = 1`` and dense
attention.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "l2_normalize",
    "route_vectors",
    "code_scores",
    "stable_topk",
    "route_codes",
    "build_inverted_index",
    "candidate_lists",
    "candidate_mask_dense",
    "group_mean_scores",
    "select_topk_index",
    "select_topk_dense",
    "key_codes_one_head",
    "query_codes_rows",
    "route_rows_one_head",
    "route",
    "sparse_attention",
    "sparse_attention_reference_gather",
    "dense_attention",
    "rope_reference",
    "module_forward",
    "float_key",
]


# ---------------------------------------------------------------------------
# Stage 1: routing projection + codebook scoring + top-b / top-a
# ---------------------------------------------------------------------------

def l2_normalize(x: np.ndarray, eps: float = 1e-12) -> np.ndarray:
    """``F.normalize(x, dim=-1)``: ``x / max(||x||_2, eps)`` (ssa/router.py:116-118)."""
    nrm = np.sqrt(np.sum(x * x, axis=-1, keepdims=True))
    return x / np.maximum(nrm, eps)


def _codebook_per_head(codebook: np.ndarray, h_kv: int) -> np.ndarray:
    """Per-KV-head codebook ``[h_kv, N_c, d_s]`` (ssa/router.py:66-68).

    A shared ``[N_c, d_s]`` codebook (the design document's form,
    ssa_design.md:67-68) is broadcast to every head.
    """
    if codebook.ndim == 2:
        return np.broadcast_to(codebook, (h_kv,) + codebook.shape)
    if codebook.shape[0] == 1 and h_kv > 1:
        return np.broadcast_to(codebook[0], (h_kv,) + codebook.shape[1:])
    assert codebook.shape[0] == h_kv, "codebook must be [h_kv,N_c,d_s] or [N_c,d_s]"
    return codebook


def route_vectors(q, k, w_qr, w_kr, dtype=np.float64):
    """Routing projection with GQA group mean (ssa/router.py:102-112).

    The reference projects every query head (``W_qr(q_full)``) and then
    averages the ``g`` projected routes of a KV group.  Returns the
    *un-normalised* routes ``q_route [n, h_kv, d_s]`` and ``k_route [n, h_kv, d_s]``.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    n, h_q, _ = q.shape
    h_kv = k.shape[1]
    assert h_q % h_kv == 0, "num_q_heads must be divisible by num_kv_heads"
    g = h_q // h_kv
    q_route = q @ np.asarray(w_qr, dtype=dtype).T          # [n, h_q, d_s]
    k_route = k @ np.asarray(w_kr, dtype=dtype).T          # [n, h_kv, d_s]
    d_s = q_route.shape[-1]
    q_route = q_route.reshape(n, h_kv, g, d_s).mean(axis=2)
    return q_route, k_route


def code_scores(route, codebook, temperature=1.0, dtype=np.float64):
    """Cosine scores ``einsum('shd,hcd->shc')/temperature`` (ssa/router.py:116-126)."""
    route = np.asarray(route, dtype=dtype)
    h_kv = route.shape[1]
    cb = l2_normalize(np.asarray(_codebook_per_head(codebook, h_kv), dtype=dtype))
    rn = l2_normalize(route)
    s = np.empty(rn.shape[:2] + (cb.shape[1],), dtype=np.result_type(rn, cb))
    for h in range(h_kv):                                   # [n, d_s] @ [d_s, N_c] per head
        s[:, h, :] = np.ascontiguousarray(rn[:, h, :]) @ cb[h].T
    return s / temperature


def stable_topk(scores: np.ndarray, kk: int) -> np.ndarray:
    """Indices of the ``kk`` largest entries along the last axis, sorted by
    score descending with the lower index first among equal scores.

    Restates ``Tensor.topk`` (ssa/router.py:130,141,204) with the oracle's
    canonical tie rule.  ``-0.0`` and ``+0.0`` compare equal.
    """
    scores = np.asarray(scores)
    n = scores.shape[-1]
    if kk >= n or n <= 64:
        order = np.argsort(-scores, axis=-1, kind="stable")
        return order[..., :kk]
    # threshold = kk-th largest value; keep every value above it and the
    # lowest-index values equal to it, then order the kk survivors.
    thr = np.partition(scores, n - kk, axis=-1)[..., n - kk:n - kk + 1]
    sel = (scores >= thr).reshape(-1, n)
    over = np.nonzero(sel.sum(axis=-1) > kk)[0]          # rows with ties across the threshold
    if over.size:
        s2 = scores.reshape(-1, n)[over]
        t2 = thr.reshape(-1, 1)[over]
        gt, eq = s2 > t2, s2 == t2
        need = kk - gt.sum(axis=-1, keepdims=True)
        sel[over] = gt | (eq & (np.cumsum(eq, axis=-1) <= need))
    cols = np.nonzero(sel)[1].reshape(scores.shape[:-1] + (kk,))
    vals = np.take_along_axis(scores, cols, axis=-1)
    order = np.argsort(-vals, axis=-1, kind="stable")     # cols ascend, so ties keep index order
    return np.take_along_axis(cols, order, axis=-1)


def route_codes(q, k, w_qr, w_kr, codebook, a, b, temperature=1.0, dtype=np.float64):
    """Stage 1: ``(q_codes [n,h_kv,a], k_codes [n,h_kv,b])`` (ssa/router.py:102-141)."""
    q_route, k_route = route_vectors(q, k, w_qr, w_kr, dtype=dtype)
    qs = code_scores(q_route, codebook, temperature, dtype=dtype)
    ks = code_scores(k_route, codebook, temperature, dtype=dtype)
    return stable_topk(qs, a), stable_topk(ks, b)


# ---------------------------------------------------------------------------
# Stage 2: candidate generation
# ---------------------------------------------------------------------------

def build_inverted_index(k_codes: np.ndarray, n_codes: int):
    """Code -> key inverted index, per KV head, keys ascending in each bucket.

    ``k_codes [n, h_kv, b]`` -> ``(bucket_ptr [h_kv, n_codes+1], bucket_keys [h_kv, n*b])``
    with bucket ``c`` of head ``h`` = ``bucket_keys[h, ptr[h,c]:ptr[h,c+1]]``.
    The reference never builds this structure; it is the linear-memory form
    of the match that ``_build_candidate_mask`` (ssa/router.py:216-259)
    evaluates densely, and of the index the design document describes
    (ssa_design.md:103-112).
    """
    n, h_kv, b = k_codes.shape
    ptr = np.zeros((h_kv, n_codes + 1), dtype=np.int64)
    keys = np.zeros((h_kv, n * b), dtype=np.int64)
    key_of = np.repeat(np.arange(n, dtype=np.int64), b)
    for h in range(h_kv):
        flat = k_codes[:, h, :].reshape(-1).astype(np.int64)
        order = np.argsort(flat, kind="stable")          # by code, then key ascending
        keys[h] = key_of[order]
        ptr[h, 1:] = np.cumsum(np.bincount(flat, minlength=n_codes))
    return ptr, keys


def candidate_lists(q_codes, k_codes, n_codes, causal=True):
    """Per (i, h) sorted unique candidate keys: keys sharing a code with the
    query, restricted to ``j <= i`` when causal.

    Equals ``_build_candidate_mask`` (ssa/router.py:216-259) ANDed with the
    causal mask (ssa/router.py:185-188).  Returns a list over heads of
    ``(row_ptr [n+1], keys)`` CSR arrays.
    """
    n, h_kv, a = q_codes.shape
    ptr, keys = build_inverted_index(k_codes, n_codes)
    out = []
    for h in range(h_kv):
        codes = q_codes[:, h, :].reshape(-1).astype(np.int64)      # [n*a]
        lo = ptr[h, codes]
        ln = ptr[h, codes + 1] - lo
        qi = np.repeat(np.repeat(np.arange(n, dtype=np.int64), a), ln)
        starts = np.repeat(lo - np.concatenate(([0], np.cumsum(ln)[:-1])), ln)
        kj = keys[h, np.arange(ln.sum(), dtype=np.int64) + starts]
        if causal:
            keep = kj <= qi
            qi, kj = qi[keep], kj[keep]
        pair = np.unique(qi * n + kj)
        qi, kj = pair // n, pair % n
        row_ptr = np.zeros(n + 1, dtype=np.int64)
        row_ptr[1:] = np.cumsum(np.bincount(qi, minlength=n))
        out.append((row_ptr, kj))
    return out


def candidate_mask_dense(q_codes, k_codes):
    """Literal restatement of ``_build_candidate_mask`` (ssa/router.py:216-259):
    ``mask[i,h,j] = any(q_codes[i,h,:] == k_codes[j,h,:])``.  O(n^2): small n only."""
    n, h_kv, a = q_codes.shape
    mask = np.zeros((n, h_kv, n), dtype=bool)
    for j0 in range(0, n, 128):
        j1 = min(j0 + 128, n)
        m = q_codes[:, None, :, None, :] == k_codes[None, j0:j1, :, :, None]
        mask[:, :, j0:j1] = m.any(axis=(-1, -2)).transpose(0, 2, 1)
    return mask


def group_mean_scores(q, k, i_rows, j_cols, h, dtype=np.float64):
    """Group-mean full-dimension logits ``mean_g(q_{i,g} . k_j) / sqrt(d)``
    for pairs ``(i_rows[p], j_cols[p])`` of KV head ``h`` (ssa/router.py:180-191)."""
    n, h_q, d = q.shape
    g = h_q // k.shape[1]
    qbar = np.asarray(q[:, h * g:(h + 1) * g, :], dtype=dtype).mean(axis=1)   # [n, d]
    kh = np.asarray(k[:, h, :], dtype=dtype)
    out = np.empty(len(i_rows), dtype=dtype)
    step = 1 << 16
    for s in range(0, len(i_rows), step):
        out[s:s + step] = np.einsum("pd,pd->p", qbar[i_rows[s:s + step]], kh[j_cols[s:s + step]])
    return out / np.sqrt(d)


def _fill_row(cands_sorted_by_score, cand_set_sorted, n, top_k):
    """Canonical top-k row: ranked candidates, then the lowest-index
    non-candidates, then zero padding when ``top_k > n`` (ssa/router.py:203-211)."""
    eff = min(top_k, n)
    row = np.zeros(top_k, dtype=np.int64)
    m = min(len(cands_sorted_by_score), eff)
    row[:m] = cands_sorted_by_score[:m]
    need = eff - m
    if need > 0:
        pool = np.arange(need + len(cand_set_sorted), dtype=np.int64)
        filler = np.setdiff1d(pool, cand_set_sorted, assume_unique=True)[:need]
        row[m:eff] = filler
    return row


def select_topk_index(q, k, q_codes, k_codes, n_codes, top_k, causal=True,
                      score_fn=None, dtype=np.float64):
    """Stage 2 through the inverted index: candidates, group-mean re-score,
    stable top-k, canonical filler, zero padding.  Returns ``[n, h_kv, top_k]``
    int64 (ssa/router.py:151-214 under the oracle's corrections).

    ``score_fn(i_rows, j_cols, h) -> scores`` overrides the re-score (used by
    the tie tests, which feed exact scores)."""
    n, h_kv, _ = k.shape
    lists = candidate_lists(q_codes, k_codes, n_codes, causal=causal)
    out = np.zeros((n, h_kv, top_k), dtype=np.int64)
    for h in range(h_kv):
        row_ptr, kj = lists[h]
        qi = np.repeat(np.arange(n, dtype=np.int64), np.diff(row_ptr))
        if score_fn is None:
            sc = group_mean_scores(q, k, qi, kj, h, dtype=dtype)
        else:
            sc = np.asarray(score_fn(qi, kj, h))
        order = np.lexsort((kj, -sc, qi))              # by query, score desc, key asc
        kj_ranked = kj[order]
        for i in range(n):
            s, e = row_ptr[i], row_ptr[i + 1]
            out[i, h] = _fill_row(kj_ranked[s:e], kj[s:e], n, top_k)
    return out


def select_topk_dense(q, k, q_codes, k_codes, top_k, causal=True, dtype=np.float64,
                      q_block=None, q_start=0):
    """Stage 2 as the reference computes it (ssa/router.py:170-214): the full
    ``[n, h_kv, g, n]`` logits, causal ``-inf``, group mean, candidate-mask
    ``-inf``, top-k over all ``n`` keys -- with the stable tie rule, which
    makes the ``-inf`` filler the lowest-index non-candidates.

    O(n^2) per head, processed in query blocks of ``q_block`` rows.  ``q``
    (and ``q_codes``) may hold a block of query rows at sequence positions
    ``q_start, q_start+1, ...`` (used by the CPU baseline's bounded sample).
    This is the CPU baseline's algorithm (the reference's own), and a
    cross-check of :func:`select_topk_index`."""
    n_q, h_q, d = q.shape
    n, h_kv = k.shape[0], k.shape[1]
    g = h_q // h_kv
    eff = min(top_k, n)
    n_codes = int(max(np.max(q_codes), np.max(k_codes))) + 1
    out = np.zeros((n_q, h_kv, top_k), dtype=np.int64)
    qb = q_block or n_q
    jj = np.arange(n)
    for h in range(h_kv):
        qh = np.asarray(q[:, h * g:(h + 1) * g, :], dtype=dtype)     # [n_q, g, d]
        kh = np.asarray(k[:, h, :], dtype=dtype)                       # [n, d]
        kc = k_codes[:, h, :]
        for i0 in range(0, n_q, qb):
            i1 = min(i0 + qb, n_q)
            full = (qh[i0:i1].reshape(-1, d) @ kh.T).reshape(i1 - i0, g, n) / np.sqrt(d)
            sc = full.mean(axis=1)                                      # [blk, n]
            if causal:
                sc[jj[None, :] > (q_start + np.arange(i0, i1))[:, None]] = -np.inf
            # mask[i, j] = any(q_codes[i] == k_codes[j]) via a per-query code-membership row
            member = np.zeros((i1 - i0, n_codes), dtype=bool)
            np.put_along_axis(member, q_codes[i0:i1, h, :].astype(np.int64), True, axis=1)
            cm = np.take_along_axis(member, np.broadcast_to(kc.reshape(1, -1), (i1 - i0, kc.size)),
                                    axis=1).reshape(i1 - i0, n, -1).any(axis=2)
            sc[~cm] = -np.inf
            out[i0:i1, h, :eff] = stable_topk(sc, eff)
    return out


def key_codes_one_head(k_head, w_kr, codebook_head, b, temperature=1.0, block=8192, dtype=np.float64):
    """Top-``b`` codes ``[n, b]`` of every key of one KV head
    (``k_head [n, d]``, ``codebook_head [N_c, d_s]``): the key half of
    ssa/router.py:102-130, in blocks of ``block`` keys so that the
    ``[block, N_c]`` score matrix is the only large temporary."""
    kr = np.asarray(k_head, dtype=dtype) @ np.asarray(w_kr, dtype=dtype).T      # [n, d_s]
    cb = l2_normalize(np.asarray(codebook_head, dtype=dtype))
    kn = l2_normalize(kr)
    out = np.empty((kn.shape[0], b), dtype=np.int64)
    for s in range(0, kn.shape[0], block):
        out[s:s + block] = stable_topk((kn[s:s + block] @ cb.T) / temperature, b)
    return out


def query_codes_rows(q_rows, w_qr, codebook_head, a, temperature=1.0, dtype=np.float64):
    """Top-``a`` codes ``[r, a]`` of query rows ``q_rows [r, g, d]`` of one KV
    group: the group mean of the per-head routes, normalised, scored against
    the normalised codebook (ssa/router.py:102-141)."""
    qr = (np.asarray(q_rows, dtype=dtype) @ np.asarray(w_qr, dtype=dtype).T).mean(axis=1)   # [r, d_s]
    cb = l2_normalize(np.asarray(codebook_head, dtype=dtype))
    return stable_topk((l2_normalize(qr) @ cb.T) / temperature, a)


def route_rows_one_head(q_rows, positions, k_head, w_qr, w_kr, codebook_head, a, b, top_k,
                        causal=True, temperature=1.0, dtype=np.float64, k_codes=None):
    """``CodebookRouter.forward`` (ssa/router.py:73-214, with the oracle's
    corrections) for a SAMPLE of query rows of one KV head, so that full
    benchmark sizes (n = 32768 .. 131072) can be checked row by row.

    ``q_rows [r, g, d]`` are the group's query heads at sequence positions
    ``positions [r]``; ``k_head [n, d]`` is every key of the head.  Each row's
    candidates are the keys ``j <= position`` (when causal) sharing one of its
    ``a`` codes (the inverted-index form of ssa/router.py:216-259), ranked by
    ``qbar . k_j`` (the group mean of the logits, ssa/router.py:180-191)
    with the lower key first among equal scores, completed with the
    lowest-index non-candidates and zero-padded past ``n`` (:func:`_fill_row`).
    Returns ``(k_codes [n, b], q_codes [r, a], indices [r, top_k])``;
    ``k_codes`` may be passed in to skip the key scoring."""
    k_head = np.asarray(k_head, dtype=dtype)
    n, d = k_head.shape
    if k_codes is None:
        k_codes = key_codes_one_head(k_head, w_kr, codebook_head, b, temperature, dtype=dtype)
    n_codes = np.asarray(codebook_head).shape[0]
    q_rows = np.asarray(q_rows, dtype=dtype)
    q_codes = query_codes_rows(q_rows, w_qr, codebook_head, a, temperature, dtype=dtype)
    ptr, keys = build_inverted_index(k_codes[:, None, :], n_codes)
    ptr, keys = ptr[0], keys[0]
    qbar = q_rows.mean(axis=1)                                    # [r, d]
    out = np.zeros((len(positions), top_k), dtype=np.int64)
    for t, pos in enumerate(positions):
        cand = np.concatenate([keys[ptr[c]:ptr[c + 1]] for c in q_codes[t]])
        cand = np.unique(cand)
        if causal:
            cand = cand[cand <= pos]
        sc = (k_head[cand] @ qbar[t]) / np.sqrt(d)
        order = np.lexsort((cand, -sc))
        out[t] = _fill_row(cand[order], cand, n, top_k)
    return k_codes, q_codes, out


def route(q, k, w_qr, w_kr, codebook, a, b, top_k, causal=True, temperature=1.0,
          dtype=np.float64, dense=False):
    """Full ``CodebookRouter.forward`` (ssa/router.py:73-149): indices ``[n,h_kv,k]`` int64."""
    q_codes, k_codes = route_codes(q, k, w_qr, w_kr, codebook, a, b, temperature, dtype)
    n_codes = np.asarray(codebook).shape[-2]
    if dense:
        return select_topk_dense(q, k, q_codes, k_codes, top_k, causal, dtype)
    return select_topk_index(q, k, q_codes, k_codes, n_codes, top_k, causal, dtype=dtype)


# ---------------------------------------------------------------------------
# Stage 3
# ---------------------------------------------------------------------------

def _softmax_attend(q_grouped, k_sel, v_sel, valid, scale):
    logits = np.matmul(q_grouped, np.swapaxes(k_sel, -1, -2)) / scale         # [n, h, g, kk]
    logits = np.where(valid[:, :, None, :], logits, -np.inf)
    m = logits.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)                   # a row with no valid key
    p = np.exp(logits - m)
    den = p.sum(axis=-1, keepdims=True)
    p /= np.where(den > 0, den, 1.0)
    return np.matmul(p, v_sel)


def sparse_attention(q, k, v, indices, scale=None, causal=False, dtype=np.float64,
                     q_offset=0, positions=None):
    """Stage 3 with the per-head gather ``k[idx, h]`` (ssa/attention.py:12-115,
    corrected).  ``scale`` divides the logits (default ``sqrt(d)``,
    ssa/attention.py:37-38,107).  ``causal`` masks keys ``j > i + q_offset``,
    or ``j > positions[i]`` when the rows of ``q`` are a sample at the
    sequence positions ``positions``.  A row with no valid key is zero (the
    reference never masks here; the build defines the empty softmax as 0).
    Duplicate indices count once per occurrence, like the reference's gather."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    n, h_q, d = q.shape
    h_kv = k.shape[1]
    g = h_q // h_kv
    if scale is None:
        scale = np.sqrt(d)
    idx = np.asarray(indices, dtype=np.int64)
    hh = np.arange(h_kv)[None, :, None]
    k_sel = k[idx, hh]                                    # [n, h_kv, kk, d]
    v_sel = v[idx, hh]
    if causal:
        pos = np.arange(n) + q_offset if positions is None else np.asarray(positions)
        valid = idx <= pos[:, None, None]
    else:
        valid = np.ones(idx.shape, dtype=bool)
    out = _softmax_attend(q.reshape(n, h_kv, g, d), k_sel, v_sel, valid, scale)
    return out.reshape(n, h_q, d)


def sparse_attention_reference_gather(q, k, v, indices, scale=None, dtype=np.float64):
    """The reference's stage 3 *including* its flattened-gather row mapping
    (``row = h*seq_len + idx`` into ``k.reshape(seq*h_kv, d)``,
    ssa/attention.py:70-100).  Used only to pin the oracle to the raw
    reference where ``h_kv > 1``."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    n, h_q, d = q.shape
    h_kv = k.shape[1]
    g = h_q // h_kv
    if scale is None:
        scale = np.sqrt(d)
    idx = np.asarray(indices, dtype=np.int64)
    rows = idx + (np.arange(h_kv) * n)[None, :, None]
    k_sel = k.reshape(n * h_kv, d)[rows]
    v_sel = v.reshape(n * h_kv, d)[rows]
    valid = np.ones(idx.shape, dtype=bool)
    return _softmax_attend(q.reshape(n, h_kv, g, d), k_sel, v_sel, valid, scale).reshape(n, h_q, d)


def dense_attention(q, k, v, causal=True, scale=None, dtype=np.float64):
    """Dense GQA attention with optional causal mask (ssa/attention.py:118-158)."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    n, h_q, d = q.shape
    h_kv = k.shape[1]
    g = h_q // h_kv
    if scale is None:
        scale = np.sqrt(d)
    ke = np.repeat(k, g, axis=1)
    ve = np.repeat(v, g, axis=1)
    logits = np.matmul(q.transpose(1, 0, 2), ke.transpose(1, 2, 0)).transpose(1, 0, 2) / scale
    if causal:
        logits = np.where(np.tril(np.ones((n, n), dtype=bool))[:, None, :], logits, -np.inf)
    m = logits.max(axis=-1, keepdims=True)
    p = np.exp(logits - m)
    p /= p.sum(axis=-1, keepdims=True)
    return np.matmul(p.transpose(1, 0, 2), ve.transpose(1, 0, 2)).transpose(1, 0, 2)


# ---------------------------------------------------------------------------
# Module level (SSAAttention)
# ---------------------------------------------------------------------------

def rope_reference(x, freqs):
    """``apply_rope`` exactly as the reference computes it (ssa/utils.py:7-48).

    The second-last axis is taken as the sequence axis, so on the
    ``[seq, heads, d]`` tensors ``SSAAttention`` passes in
    (ssa/ssa_layer.py:115-117) the rotation angle follows the *head* index;
    only the first ``d/2`` features rotate, with ``rotate_half`` pairing
    ``(t, t + d/4)``."""
    x = np.asarray(x, dtype=np.float64)
    rows, d = x.shape[-2], x.shape[-1]
    half = d // 2
    f = np.asarray(freqs, dtype=np.float64)[:rows, :half]
    cos, sin = np.cos(f), np.sin(f)
    xr, xp = x[..., :half], x[..., half:]
    q4 = half // 2
    rot = np.concatenate([-xr[..., q4:], xr[..., :q4]], axis=-1)
    return np.concatenate([xr * cos + rot * sin, xp], axis=-1)


def module_forward(x, weights, h_q, h_kv, d, n_codes, a, b, top_k, freqs=None,
                   position_ids=None, temperature=1.0, indices=None, return_attn=False):
    """``SSAAttention.forward`` (ssa/ssa_layer.py:68-138) with the oracle's
    corrections: projections, per-batch RoPE quirk, router, stage 3 with the
    causal mask, ``o_proj``.  ``weights`` maps the reference state_dict keys
    (``q_proj.weight`` ... ``router.codebook``) to arrays.

    ``indices [B, n, h_kv, k]``, if given, replace the router's selection (to
    check stage 3 and ``o_proj`` on another implementation's selection);
    ``return_attn`` adds the stage-3 output ``[B, n, h_q, d]`` (the input of
    ``o_proj``) to the result."""
    x = np.asarray(x, dtype=np.float64)
    bsz, n, _ = x.shape
    w = {kk: np.asarray(v, dtype=np.float64) for kk, v in weights.items()}
    q = (x @ w["q_proj.weight"].T).reshape(bsz, n, h_q, d)
    k = (x @ w["k_proj.weight"].T).reshape(bsz, n, h_kv, d)
    v = (x @ w["v_proj.weight"].T).reshape(bsz, n, h_kv, d)
    outs, idxs = [], []
    for bi in range(bsz):
        qb, kb = q[bi], k[bi]
        if freqs is not None:
            fb = freqs[position_ids[bi]] if position_ids is not None else freqs[:n]
            qb, kb = rope_reference(qb, fb), rope_reference(kb, fb)
        if indices is None:
            idx = route(qb, kb, w["router.W_qr.weight"], w["router.W_kr.weight"],
                        w["router.codebook"], a, b, top_k, causal=True, temperature=temperature)
        else:
            idx = np.asarray(indices[bi], dtype=np.int64)
        idxs.append(idx)
        outs.append(sparse_attention(qb, kb, v[bi], idx, causal=True))
    attn = np.stack(outs)
    y = attn.reshape(bsz, n, h_q * d) @ w["o_proj.weight"].T
    if return_attn:
        return y, np.stack(idxs), attn
    return y, np.stack(idxs)


# ---------------------------------------------------------------------------
# helpers for tie-aware comparisons
# ---------------------------------------------------------------------------

def float_key(x: np.ndarray) -> np.ndarray:
    """Order-preserving uint32 key of float32 values (``-0.0`` folded into ``+0.0``)."""
    x = np.asarray(x, dtype=np.float32) + np.float32(0.0)
    u = x.view(np.uint32)
    return np.where(u >> 31, ~u, u | np.uint32(0x80000000)).astype(np.uint32)
