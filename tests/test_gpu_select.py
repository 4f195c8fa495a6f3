"""Bit-exact parity of the selection stages on the GPU (fed inputs).

* code selection (top-a / top-b) on fed fp32 scores with forced ties;
* the code->key inverted index;
* candidate union + causal filter + re-score + top-k + filler, on
  integer-valued q/k so that every score is exact in fp32 and ties are
  common -- the lowest-index tie rule is checked exactly.
"""

import numpy as np
import pytest
import torch

from oracle import ssa_oracle as O
from ssa_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("rows,n_cols,kk", [(257, 64, 4), (300, 4096, 16), (64, 5000, 32), (33, 9, 8)])
def test_select_from_scores_ties(rows, n_cols, kk):
    rng = np.random.default_rng(rows + n_cols)
    s = (rng.integers(-6, 7, size=(rows, n_cols)) / 4.0).astype(np.float32)
    zeros = s == 0
    s[zeros & (rng.random(s.shape) < 0.5)] = -0.0          # -0.0 ties +0.0
    got = ops.select_from_scores(torch.from_numpy(s).to(DEV), kk).cpu().numpy()
    np.testing.assert_array_equal(got, O.stable_topk(s, kk))


def test_select_from_scores_random_fp32():
    rng = np.random.default_rng(3)
    s = rng.standard_normal((1000, 4096)).astype(np.float32)
    got = ops.select_from_scores(torch.from_numpy(s).to(DEV), 16).cpu().numpy()
    np.testing.assert_array_equal(got, O.stable_topk(s, 16))


def _distinct_codes(rng, shape, n_codes, per):
    """[..., per] distinct codes per row (like top-k indices)."""
    r = rng.random(shape + (n_codes,))
    return np.argsort(r, axis=-1)[..., :per].astype(np.int32)


@pytest.mark.parametrize("B,n,h_kv,b,n_codes", [(1, 1, 1, 1, 16), (2, 100, 3, 4, 16), (1, 5000, 2, 4, 4096),
                                                 (1, 3000, 1, 7, 64), (1, 9000, 2, 4, 32)])
def test_inverted_index_bit_exact(B, n, h_kv, b, n_codes):
    rng = np.random.default_rng(n + b)
    kc = _distinct_codes(rng, (B, n, h_kv), n_codes, b)
    ptr, keys = ops.build_index(torch.from_numpy(kc).to(DEV), n_codes)
    ptr, keys = ptr.cpu().numpy(), keys.cpu().numpy()
    for bi in range(B):
        eptr, ekeys = O.build_inverted_index(kc[bi], n_codes)
        np.testing.assert_array_equal(ptr[bi], eptr)
        np.testing.assert_array_equal(keys[bi], ekeys)


def _int_inputs(rng, n, h_q, h_kv, d, dtype, B=1):
    q = rng.integers(-2, 3, size=(B, n, h_q, d)).astype(np.float32)
    k = rng.integers(-2, 3, size=(B, n, h_kv, d)).astype(np.float32)
    return q, k, torch.from_numpy(q).to(DEV, dtype), torch.from_numpy(k).to(DEV, dtype)


CASES = [
    # n, h_q, h_kv, d, n_codes, a, b, top_k, causal
    (64, 4, 1, 16, 16, 4, 2, 8, True),
    (300, 8, 2, 64, 32, 8, 4, 16, True),
    (300, 8, 2, 64, 32, 8, 4, 16, False),
    (50, 4, 2, 32, 8, 2, 2, 80, True),          # k > n: zero padding
    (50, 4, 2, 32, 8, 2, 2, 50, True),          # k == n
    (1000, 4, 1, 128, 512, 16, 4, 64, True),    # sparse: most rows need filler
    (5000, 2, 1, 32, 4, 2, 2, 64, True),        # > 2048 candidates: radix-select path
    (700, 16, 2, 128, 64, 16, 4, 256, True),
    (1500, 4, 1, 64, 32, 4, 2, 300, True),      # 257..512 candidates: 16-per-lane warp sort
    (600, 8, 2, 64, 16, 4, 2, 600, True),       # k > 512: every unit on the CTA-wide path
    (400, 4, 1, 64, 64, 32, 4, 32, True),       # a = 32 query codes
    (3000, 4, 1, 64, 16, 4, 4, 64, True),       # up to ~2200 candidates: every warp tier, then the CTA path
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", CASES)
def test_select_candidates_bit_exact(case, dtype):
    n, h_q, h_kv, d, n_codes, a, b, top_k, causal = case
    rng = np.random.default_rng(n * 7 + top_k)
    qn, kn, q, k = _int_inputs(rng, n, h_q, h_kv, d, dtype)
    qc = _distinct_codes(rng, (1, n, h_kv), n_codes, a)
    kc = _distinct_codes(rng, (1, n, h_kv), n_codes, b)
    idx, counts = ops.select_candidates(q, k, torch.from_numpy(qc).to(DEV), torch.from_numpy(kc).to(DEV),
                                        n_codes, top_k, causal=causal)
    expect = O.select_topk_index(qn[0], kn[0], qc[0], kc[0], n_codes, top_k, causal=causal)
    np.testing.assert_array_equal(idx[0].cpu().numpy(), expect)
    lists = O.candidate_lists(qc[0], kc[0], n_codes, causal=causal)
    for h in range(h_kv):
        np.testing.assert_array_equal(counts[0, :, h].cpu().numpy(), np.diff(lists[h][0]))


def test_select_candidates_query_shard_and_int32():
    n, h_q, h_kv, d, n_codes, a, b, top_k = 400, 8, 2, 64, 32, 8, 4, 32
    rng = np.random.default_rng(11)
    qn, kn, q, k = _int_inputs(rng, n, h_q, h_kv, d, torch.float32)
    qc = _distinct_codes(rng, (1, n, h_kv), n_codes, a)
    kc = _distinct_codes(rng, (1, n, h_kv), n_codes, b)
    expect = O.select_topk_index(qn[0], kn[0], qc[0], kc[0], n_codes, top_k, causal=True)
    lo, hi = 150, 290
    idx, _ = ops.select_candidates(q[:, lo:hi], k, torch.from_numpy(qc[:, lo:hi]).to(DEV),
                                   torch.from_numpy(kc).to(DEV), n_codes, top_k, causal=True,
                                   q_offset=lo, index_i64=False)
    assert idx.dtype == torch.int32
    np.testing.assert_array_equal(idx[0].cpu().numpy(), expect[lo:hi])


def test_select_candidates_batched():
    n, h_q, h_kv, d, n_codes, a, b, top_k, B = 200, 4, 2, 32, 16, 4, 2, 24, 3
    rng = np.random.default_rng(12)
    qn, kn, q, k = _int_inputs(rng, n, h_q, h_kv, d, torch.bfloat16, B=B)
    qc = _distinct_codes(rng, (B, n, h_kv), n_codes, a)
    kc = _distinct_codes(rng, (B, n, h_kv), n_codes, b)
    idx, _ = ops.select_candidates(q, k, torch.from_numpy(qc).to(DEV), torch.from_numpy(kc).to(DEV),
                                   n_codes, top_k, causal=True)
    for bi in range(B):
        expect = O.select_topk_index(qn[bi], kn[bi], qc[bi], kc[bi], n_codes, top_k, causal=True)
        np.testing.assert_array_equal(idx[bi].cpu().numpy(), expect)
