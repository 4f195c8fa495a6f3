"""Pin the CPU oracle to the reference implementation's own outputs.

The fixtures under ``tests/golden/`` were produced by running the unmodified
reference (chenxingqiang/SSA) with ``tests/golden/make_golden.py``.  These
tests need no GPU.
"""

import os

import numpy as np
import pytest

from oracle import ssa_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


def test_stage1_codes_match_reference():
    z = _load("stage1.npz")
    n, h_q, h_kv, d, d_s, n_c, a, b, k = z["dims"]
    q_route, k_route = O.route_vectors(z["q"], z["k"], z["w_qr"], z["w_kr"])
    qs = O.code_scores(q_route, z["codebook"])
    np.testing.assert_allclose(qs, z["q_code_scores"], atol=2e-6)
    q_codes = O.stable_topk(qs, a)
    k_codes = O.stable_topk(O.code_scores(k_route, z["codebook"]), b)
    np.testing.assert_array_equal(q_codes, z["top_q_codes"])
    np.testing.assert_array_equal(k_codes, z["k_code_assign"])


def test_candidate_mask_matches_reference():
    z = _load("stage1.npz")
    n, h_q, h_kv, d, d_s, n_c, a, b, k = z["dims"]
    ref = np.unpackbits(z["candidate_mask"])[: n * h_kv * n].reshape(n, h_kv, n).astype(bool)
    mine = O.candidate_mask_dense(z["top_q_codes"], z["k_code_assign"])
    np.testing.assert_array_equal(mine, ref)
    # the inverted-index restatement gives the same sets, causal-filtered
    lists = O.candidate_lists(z["top_q_codes"], z["k_code_assign"], n_c, causal=True)
    causal = np.tril(np.ones((n, n), dtype=bool))
    for h in range(h_kv):
        ptr, keys = lists[h]
        for i in range(n):
            expect = np.nonzero(ref[i, h] & causal[i])[0]
            np.testing.assert_array_equal(keys[ptr[i]:ptr[i + 1]], expect)


def test_topk_matches_reference_on_well_defined_rows():
    z = _load("stage1.npz")
    n, h_q, h_kv, d, d_s, n_c, a, b, k = z["dims"]
    mine = O.select_topk_index(z["q"], z["k"], z["top_q_codes"], z["k_code_assign"], n_c, k,
                               causal=True)
    wd = z["well_defined"]
    assert wd.sum() > 100
    np.testing.assert_array_equal(mine[wd], z["indices"][wd])
    dense = O.select_topk_dense(z["q"], z["k"], z["top_q_codes"], z["k_code_assign"], k,
                                causal=True, q_block=32)
    np.testing.assert_array_equal(dense, mine)


@pytest.mark.parametrize("scale_key,scale", [("out", None), ("out_scale", 2.5)])
def test_stage3_single_kv_head_matches_reference(scale_key, scale):
    z = _load("stage3_h1.npz")
    out = O.sparse_attention(z["q"], z["k"], z["v"], z["indices"], scale=scale, causal=False)
    np.testing.assert_allclose(out, z[scale_key], rtol=1e-5, atol=1e-5)


def test_stage3_gqa_gather_bug_is_pinned():
    """At h_kv = 2 the raw reference follows its flattened row mapping; the
    oracle's corrected per-head gather differs from it."""
    z = _load("stage3_h2.npz")
    raw = O.sparse_attention_reference_gather(z["q"], z["k"], z["v"], z["indices"])
    np.testing.assert_allclose(raw, z["out"], rtol=1e-5, atol=1e-5)
    fixed = O.sparse_attention(z["q"], z["k"], z["v"], z["indices"], causal=False)
    assert np.abs(fixed - z["out"]).max() > 1e-2


def test_dense_matches_reference():
    z = _load("dense.npz")
    out = O.dense_attention(z["q"], z["k"], z["v"], causal=True)
    np.testing.assert_allclose(out, z["out"], rtol=1e-5, atol=1e-5)


def _module_weights(z):
    return {kname[3:].replace("__", "."): z[kname] for kname in z.files if kname.startswith("sd_")}


def test_module_rope_quirk_and_output_match_reference():
    z = _load("module.npz")
    hs, h_q, h_kv, d, n, d_s, n_c, b, a, k = z["dims"]
    w = _module_weights(z)
    x = z["x"][0].astype(np.float64)
    q = (x @ w["q_proj.weight"].T.astype(np.float64)).reshape(n, h_q, d)
    kk = (x @ w["k_proj.weight"].T.astype(np.float64)).reshape(n, h_kv, d)
    np.testing.assert_allclose(O.rope_reference(q, z["freqs"][:n]), z["q_rope"], atol=2e-5)
    np.testing.assert_allclose(O.rope_reference(kk, z["freqs"][:n]), z["k_rope"], atol=2e-5)
    y, idx = O.module_forward(z["x"], w, h_q, h_kv, d, n_c, a, b, k, freqs=z["freqs"])
    rows = z["well_defined_rows"]
    assert rows.sum() > 40
    np.testing.assert_array_equal(idx[0][rows], z["indices"][rows])
    np.testing.assert_allclose(y[0][rows], z["y"][0][rows], rtol=1e-4, atol=1e-5)


def test_k_equals_n_reproduces_dense_causal():
    rng = np.random.default_rng(5)
    n, h_q, h_kv, d = 64, 6, 2, 16
    q = rng.standard_normal((n, h_q, d))
    k = rng.standard_normal((n, h_kv, d))
    v = rng.standard_normal((n, h_kv, d))
    w_qr = rng.standard_normal((8, d))
    w_kr = rng.standard_normal((8, d))
    cb = rng.standard_normal((h_kv, 32, 8))
    idx = O.route(q, k, w_qr, w_kr, cb, a=4, b=2, top_k=n, causal=True)
    for h in range(h_kv):
        for i in range(n):
            assert sorted(idx[i, h].tolist()) == list(range(n))
    out = O.sparse_attention(q, k, v, idx, causal=True)
    np.testing.assert_allclose(out, O.dense_attention(q, k, v, causal=True), atol=1e-12)


def test_zero_padding_when_k_exceeds_n():
    rng = np.random.default_rng(6)
    n, h_q, h_kv, d = 10, 4, 2, 8
    q = rng.standard_normal((n, h_q, d))
    k = rng.standard_normal((n, h_kv, d))
    idx = O.route(q, k, rng.standard_normal((4, d)), rng.standard_normal((4, d)),
                  rng.standard_normal((h_kv, 8, 4)), a=2, b=2, top_k=16, causal=True)
    assert idx.shape == (n, h_kv, 16)
    assert (idx[:, :, n:] == 0).all()
    for h in range(h_kv):
        for i in range(n):
            assert sorted(idx[i, h, :n].tolist()) == list(range(n))


def test_torch_port_matches_oracle_on_tie_free_rows():
    """The torch-CPU port timed as the CPU baseline computes the oracle's
    result wherever the selection is well defined (rows with at least k
    candidates; random inputs have no ties)."""
    import torch

    from oracle import ssa_port_torch as P

    rng = np.random.default_rng(21)
    n, h_q, h_kv, d, d_s, n_c, a, b, kk = 300, 8, 2, 32, 8, 64, 4, 2, 24
    g = h_q // h_kv
    q = rng.standard_normal((n, h_q, d))
    k = rng.standard_normal((n, h_kv, d))
    v = rng.standard_normal((n, h_kv, d))
    w_qr = rng.standard_normal((d_s, d)) / np.sqrt(d)
    w_kr = rng.standard_normal((d_s, d)) / np.sqrt(d)
    cb = rng.standard_normal((h_kv, n_c, d_s))
    qc_o, kc_o = O.route_codes(q, k, w_qr, w_kr, cb, a, b)
    idx_o = O.select_topk_dense(q, k, qc_o, kc_o, kk, causal=True)
    out_o = O.sparse_attention(q, k, v, idx_o, causal=True)
    counts = O.candidate_mask_dense(qc_o, kc_o)
    T = lambda x: torch.from_numpy(np.ascontiguousarray(x))
    for h in range(h_kv):
        qh, kh, vh = T(q[:, h * g:(h + 1) * g]), T(k[:, h]), T(v[:, h])
        kc = P.key_codes(kh, T(w_kr), T(cb[h]), b)
        qc = P.query_codes(qh, T(w_qr), T(cb[h]), a)
        np.testing.assert_array_equal(kc.numpy(), kc_o[:, h])
        np.testing.assert_array_equal(qc.numpy(), qc_o[:, h])
        idx = P.select(qh, kh, qc, kc, n_c, kk, 0, True, block=64).numpy()
        causal_cands = (counts[:, h, :] & (np.arange(n)[None, :] <= np.arange(n)[:, None])).sum(axis=1)
        full = causal_cands >= kk
        assert full.sum() > 50
        np.testing.assert_array_equal(idx[full], idx_o[full, h])
        out = P.attention(qh, kh, vh, T(idx_o[:, h]), 0, True, block=100).numpy()
        np.testing.assert_allclose(out, out_o[:, h * g:(h + 1) * g], rtol=1e-10, atol=1e-10)


def test_sampled_row_router_matches_the_full_oracle():
    """route_rows_one_head (the per-head, sampled-row form the GPU tests use
    at full benchmark sizes) equals route_codes + select_topk_index on every
    row it is given, for causal and non-causal routing, g = 3, k > candidates."""
    rng = np.random.default_rng(17)
    n, h_q, h_kv, d, d_s, n_c, a, b, k = 300, 6, 2, 32, 8, 64, 6, 3, 40
    q = rng.standard_normal((n, h_q, d))
    kk = rng.standard_normal((n, h_kv, d))
    w_qr = rng.standard_normal((d_s, d))
    w_kr = rng.standard_normal((d_s, d))
    cb = rng.standard_normal((h_kv, n_c, d_s))
    q_codes, k_codes = O.route_codes(q, kk, w_qr, w_kr, cb, a, b)
    g = h_q // h_kv
    rows = np.array([0, 1, 7, 50, 151, 298, 299])
    for causal in (True, False):
        full = O.select_topk_index(q, kk, q_codes, k_codes, n_c, k, causal=causal)
        for h in range(h_kv):
            kc, qc, idx = O.route_rows_one_head(q[rows, h * g:(h + 1) * g], rows, kk[:, h], w_qr, w_kr, cb[h],
                                                a, b, k, causal=causal)
            np.testing.assert_array_equal(kc, k_codes[:, h])
            np.testing.assert_array_equal(qc, q_codes[rows, h])
            np.testing.assert_array_equal(idx, full[rows, h])


def test_sampled_rows_of_stage3_match_the_full_rows():
    rng = np.random.default_rng(18)
    n, h_q, h_kv, d, k = 50, 4, 2, 16, 9
    q, kk, v = (rng.standard_normal((n, h, d)) for h in (h_q, h_kv, h_kv))
    idx = rng.integers(0, n, size=(n, h_kv, k))
    full = O.sparse_attention(q, kk, v, idx, causal=True)
    rows = np.array([0, 3, 20, 49])
    part = O.sparse_attention(q[rows], kk, v, idx[rows], causal=True, positions=rows)
    np.testing.assert_allclose(part, full[rows], rtol=1e-12, atol=1e-12)
    # row 0 with every index in the future has no valid key: a zero row
    idx0 = idx.copy()
    idx0[0] = n - 1
    z = O.sparse_attention(q, kk, v, idx0, causal=True)
    assert np.all(z[0] == 0) and np.isfinite(z).all()
