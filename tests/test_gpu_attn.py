"""Stage 3 (sparse exact attention) on the GPU against the oracle.

Tolerances are those of tests/_tol.py (fp32: 1e-5; bf16/fp16: 2e-3 relative
in the L2 norm and one output rounding per element).  The reference is
computed in float64 from the same (rounded) inputs.
"""

import math
import os

import numpy as np
import pytest
import torch

import ssa_b200 as ssa
from oracle import ssa_oracle as O
from _tol import assert_output_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _close(out, ref, dtype):
    assert_output_close(out, ref, dtype)


def _inputs(rng, n, h_q, h_kv, d, kk, dtype, B=1, n_keys=None):
    n_keys = n_keys or n
    qn = rng.standard_normal((B, n, h_q, d)).astype(np.float32)
    kn = rng.standard_normal((B, n_keys, h_kv, d)).astype(np.float32)
    vn = rng.standard_normal((B, n_keys, h_kv, d)).astype(np.float32)
    idx = rng.integers(0, n_keys, size=(B, n, h_kv, kk))
    t = [torch.from_numpy(x).to(DEV, dtype) for x in (qn, kn, vn)]
    # the oracle sees exactly the rounded values
    qn, kn, vn = (x.double().cpu().numpy() for x in t)
    return qn, kn, vn, idx, t


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,h_q,h_kv,d,kk,causal", [
    (64, 4, 1, 8, 8, False),
    (200, 6, 2, 16, 7, True),          # g = 3
    (300, 8, 2, 64, 256, True),
    (128, 28, 4, 128, 64, True),       # g = 7 (Qwen-style)
    (96, 32, 8, 128, 33, False),
    (64, 16, 1, 256, 5, True),         # g = 16, d = 256
    (40, 4, 4, 96, 300, False),        # k > n: duplicates
    (80, 12, 1, 128, 48, True),        # g = 12: two head tiles on the tensor-core path
    (70, 16, 1, 64, 20, False),        # g = 16, d = 64
    (50, 8, 1, 128, 17, True),         # g = 8: one full head tile
    (33, 2, 2, 64, 1, True),           # g = 1, k = 1
])
def test_sparse_attention_matches_oracle(n, h_q, h_kv, d, kk, causal, dtype):
    rng = np.random.default_rng(n + d + kk)
    qn, kn, vn, idx, (q, k, v) = _inputs(rng, n, h_q, h_kv, d, kk, dtype)
    if causal:   # keep at least one valid key per row, as the router's output always does
        idx[..., 0] = rng.integers(0, np.arange(n) + 1)[None, :, None]
    out = ssa.sparse_exact_attention(q[0], k[0], v[0], torch.from_numpy(idx[0]).to(DEV), is_causal=causal)
    ref = O.sparse_attention(qn[0], kn[0], vn[0], idx[0], causal=causal)
    assert out.dtype == dtype and out.shape == q[0].shape
    _close(out, ref, dtype)


def test_sparse_attention_batched_int32_scale_and_offset():
    rng = np.random.default_rng(5)
    B, n, h_q, h_kv, d, kk = 3, 120, 8, 2, 64, 40
    qn, kn, vn, idx, (q, k, v) = _inputs(rng, n, h_q, h_kv, d, kk, torch.float32, B=B, n_keys=300)
    off = 180
    idx[..., 0] = rng.integers(0, off + np.arange(n) + 1)[None, :, None]
    it = torch.from_numpy(idx).to(DEV, torch.int32)
    out = ssa.sparse_exact_attention(q, k, v, it, scale=3.0, is_causal=True, q_offset=off)
    for bi in range(B):
        ref = O.sparse_attention(qn[bi], kn[bi], vn[bi], idx[bi], scale=3.0, causal=True, q_offset=off)
        _close(out[bi], ref, torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_sparse_attention_batched_int32_offset_16bit(dtype):
    rng = np.random.default_rng(15)
    B, n, h_q, h_kv, d, kk = 2, 90, 16, 2, 128, 70
    qn, kn, vn, idx, (q, k, v) = _inputs(rng, n, h_q, h_kv, d, kk, dtype, B=B, n_keys=400)
    off = 250
    idx[..., 0] = rng.integers(0, off + np.arange(n) + 1)[None, :, None]
    it = torch.from_numpy(idx).to(DEV, torch.int32)
    out = ssa.sparse_exact_attention(q, k, v, it, scale=5.0, is_causal=True, q_offset=off)
    for bi in range(B):
        ref = O.sparse_attention(qn[bi], kn[bi], vn[bi], idx[bi], scale=5.0, causal=True, q_offset=off)
        _close(out[bi], ref, dtype)


def test_sparse_attention_strided_inputs():
    rng = np.random.default_rng(6)
    n, h_q, h_kv, d, kk = 100, 8, 2, 64, 16
    qn, kn, vn, idx, (q, k, v) = _inputs(rng, n, h_q, h_kv, d, kk, torch.float32)
    big = torch.zeros(1, n, h_q + 4, d + 8, device=DEV)
    big[:, :, :h_q, :d] = q
    qs = big[:, :, :h_q, :d]                       # non-contiguous rows, unit last stride
    out = ssa.sparse_exact_attention(qs[0], k[0], v[0], torch.from_numpy(idx[0]).to(DEV))
    _close(out, O.sparse_attention(qn[0], kn[0], vn[0], idx[0]), torch.float32)


@pytest.mark.parametrize("scale_key,scale", [("out", None), ("out_scale", 2.5)])
def test_sparse_attention_matches_reference_fixture(scale_key, scale):
    z = np.load(os.path.join(GOLD, "stage3_h1.npz"))
    t = {kk: torch.from_numpy(z[kk]).to(DEV) for kk in ("q", "k", "v", "indices")}
    out = ssa.sparse_exact_attention(t["q"], t["k"], t["v"], t["indices"], scale=scale)
    np.testing.assert_allclose(out.cpu().numpy(), z[scale_key], rtol=1e-5, atol=1e-5)


def test_out_of_range_index_raises():
    q = torch.randn(8, 4, 16, device=DEV)
    k = torch.randn(8, 2, 16, device=DEV)
    idx = torch.zeros(8, 2, 4, dtype=torch.long, device=DEV)
    idx[3, 1, 2] = 8
    # the device status word is read lazily: the error comes at check_errors()
    # (or at a later op call), without a host synchronisation after the op
    with pytest.raises(IndexError):
        ssa.sparse_exact_attention(q, k, k, idx)
        ssa.check_errors()
    ssa.check_errors()                                    # nothing left pending


def test_out_of_range_index_raises_at_the_next_op_call():
    q = torch.randn(8, 4, 16, device=DEV)
    k = torch.randn(8, 2, 16, device=DEV)
    idx = torch.zeros(8, 2, 4, dtype=torch.long, device=DEV)
    idx[0, 0, 0] = -3
    ssa.sparse_exact_attention(q, k, k, idx)
    torch.cuda.synchronize()
    with pytest.raises(IndexError):
        ssa.sparse_exact_attention(q, k, k, torch.zeros_like(idx))
    ssa.check_errors()


def test_sync_mode_raises_in_the_failing_call(monkeypatch):
    monkeypatch.setenv("SSA_CHECKED", "sync")
    q = torch.randn(8, 4, 16, device=DEV)
    k = torch.randn(8, 2, 16, device=DEV)
    idx = torch.zeros(8, 2, 4, dtype=torch.long, device=DEV)
    idx[5, 0, 1] = 99
    with pytest.raises(IndexError):
        ssa.sparse_exact_attention(q, k, k, idx)
    monkeypatch.setenv("SSA_CHECKED", "0")              # no status word at all
    ssa.sparse_exact_attention(q, k, k, idx)
    ssa.check_errors()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fully_masked_rows_are_zero(dtype):
    """With is_causal=True a row whose indices all lie after its position has
    no valid key; its output is a zero row (no NaN), other rows are unchanged,
    and its gradient is zero."""
    rng = np.random.default_rng(21)
    n, h_q, h_kv, d, kk = 64, 8, 2, 128, 16
    qn, kn, vn, idx, (q, k, v) = _inputs(rng, n, h_q, h_kv, d, kk, dtype)
    idx[..., 0] = rng.integers(0, np.arange(n) + 1)[None, :, None]
    dead = [(3, 0), (10, 1), (40, 0)]
    for i, h in dead:
        idx[0, i, h] = rng.integers(i + 1, n, size=kk)
    it = torch.from_numpy(idx[0]).to(DEV)
    out = ssa.sparse_exact_attention(q[0], k[0], v[0], it, is_causal=True)
    g = h_q // h_kv
    for i, h in dead:
        assert torch.count_nonzero(out[i, h * g:(h + 1) * g]) == 0
    assert torch.isfinite(out).all()
    keep = np.ones((n, h_q), dtype=bool)
    for i, h in dead:
        keep[i, h * g:(h + 1) * g] = False
    ref = O.sparse_attention(qn[0], kn[0], vn[0], idx[0], causal=True)
    _close(out.cpu()[torch.from_numpy(keep)], ref[keep], dtype)
    # backward: the dead rows get a zero gradient, everything stays finite
    qg = q[0].clone().requires_grad_()
    o = ssa.sparse_exact_attention(qg, k[0], v[0], it, is_causal=True)
    o.float().sum().backward()
    assert torch.isfinite(qg.grad).all()
    for i, h in dead:
        assert torch.count_nonzero(qg.grad[i, h * g:(h + 1) * g]) == 0


def test_out_of_range_index_raises_on_the_tensor_core_path():
    q = torch.randn(40, 8, 128, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(40, 2, 128, device=DEV, dtype=torch.bfloat16)
    idx = torch.zeros(40, 2, 24, dtype=torch.long, device=DEV)
    for bad in (-1, 40):
        idx[17, 1, 20] = bad
        with pytest.raises(IndexError):
            ssa.sparse_exact_attention(q, k, k, idx)
            ssa.check_errors()


def test_deterministic():
    rng = np.random.default_rng(8)
    _, _, _, idx, (q, k, v) = _inputs(rng, 500, 32, 8, 128, 256, torch.bfloat16)
    it = torch.from_numpy(idx[0]).to(DEV)
    a = ssa.sparse_exact_attention(q[0], k[0], v[0], it, is_causal=False)
    b = ssa.sparse_exact_attention(q[0], k[0], v[0], it, is_causal=False)
    assert torch.equal(a, b)
