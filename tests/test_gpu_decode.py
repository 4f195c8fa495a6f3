"""Token-by-token decoding (ssa_b200.decode.DecodeCache) against the
full-sequence forward.

Every per-row computation of a decode step (the key's codes, the query's
codes, candidates, re-score, top-k, attention) is the one the full forward
does for that row, so from position top_k - 1 on (where the full forward's
filler keys are all in the past) the outputs are identical.  The cache's
code->key index is updated in place (one append per step); it is rebuilt only
when a bucket could run out of free slots.
"""

import ctypes

import pytest
import torch

import ssa_b200 as ssa
from ssa_b200 import _lib as L
from ssa_b200 import ops
from ssa_b200.decode import DecodeCache

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(dtype, b, n_codes=256, B=2, n=96, h_q=8, h_kv=2, d=64, top_k=16, seed=1):
    torch.manual_seed(0)
    router = ssa.CodebookRouter(head_dim=d, route_dim=32, num_kv_heads=h_kv, num_codebook=n_codes,
                                codes_per_key=b, codes_per_query=8, top_k=top_k).to(DEV)
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn((B, n, h_q, d), generator=g).to(DEV, dtype)
    k = torch.randn((B, n, h_kv, d), generator=g).to(DEV, dtype)
    v = torch.randn((B, n, h_kv, d), generator=g).to(DEV, dtype)
    idx = router.route(q, k, causal=True)[0]
    full = ssa.sparse_exact_attention(q, k, v, idx, is_causal=True)
    return router, q, k, v, full


@pytest.mark.parametrize("dtype,b", [(torch.bfloat16, 4), (torch.float32, 4), (torch.bfloat16, 3)])
def test_decode_steps_match_the_full_forward(dtype, b):
    B, n, h_q, h_kv, d = 2, 96, 8, 2, 64
    router, q, k, v, full = _setup(dtype, b)
    cache = DecodeCache(router, B, capacity=128, num_q_heads=h_q, dtype=dtype, device=DEV)
    p0 = 20
    cache.append(k[:, :p0], v[:, :p0])
    assert torch.equal(cache.codes[:, :p0], router.key_codes(k[:, :p0]))
    for p in range(p0, n):
        out = cache.step(q[:, p:p + 1], k[:, p:p + 1], v[:, p:p + 1])
        assert out.shape == (B, 1, h_q, d)
        assert torch.equal(out, full[:, p:p + 1]), p
    ssa.check_errors()
    assert cache.n == n
    # the first append builds the index; the 76 steps append to it
    assert cache.rebuilds <= 3, cache.rebuilds
    with pytest.raises(ValueError, match="full"):
        cache.append(torch.empty((B, 40, h_kv, d), device=DEV, dtype=dtype),
                     torch.empty((B, 40, h_kv, d), device=DEV, dtype=dtype))


def test_decode_rebuilds_when_buckets_fill_and_stays_exact():
    """slack = 1 and a small codebook: buckets fill after a step or two, so
    the cache must rebuild often; every step still equals the full forward."""
    B, n, h_q = 1, 160, 8
    router, q, k, v, full = _setup(torch.bfloat16, 4, n_codes=16, B=B, n=n, top_k=24, seed=3)
    cache = DecodeCache(router, B, capacity=n, num_q_heads=h_q, dtype=torch.bfloat16, device=DEV, slack=1)
    cache.append(k[:, :30], v[:, :30])
    for p in range(30, n):
        out = cache.step(q[:, p:p + 1], k[:, p:p + 1], v[:, p:p + 1])
        assert torch.equal(out, full[:, p:p + 1]), p
    ssa.check_errors()
    assert cache.rebuilds > 1


def test_decode_index_matches_the_packed_index():
    """After a build and a run of appends, every bucket of the slotted index
    holds exactly the keys of the packed index, in the same (ascending) order."""
    B, n, h_kv, b, n_codes = 2, 700, 3, 4, 64
    router = ssa.CodebookRouter(head_dim=64, route_dim=32, num_kv_heads=h_kv, num_codebook=n_codes,
                                codes_per_key=b, codes_per_query=8, top_k=16).to(DEV)
    cache = DecodeCache(router, B, capacity=1024, num_q_heads=6, dtype=torch.bfloat16, device=DEV, slack=8)
    kk = torch.randn((B, n, h_kv, 64), device=DEV, dtype=torch.bfloat16)
    cache.append(kk[:, :500], kk[:, :500])
    for p in range(500, n):
        cache.append(kk[:, p:p + 1], kk[:, p:p + 1])
    ssa.check_errors()
    ptr, keys = ops.build_index(cache.codes[:, :n].contiguous(), n_codes)
    start, end = cache.ix_start.cpu(), cache.ix_end.cpu()
    ik, ic = cache.ix_keys.cpu(), cache.ix_codes.cpu()
    ptr, keys, codes = ptr.cpu(), keys.cpu(), cache.codes[:, :n].cpu()
    for bi in range(B):
        for h in range(h_kv):
            for c in range(n_codes):
                got = ik[bi, h, start[bi, h, c]:end[bi, h, c]]
                ref = keys[bi, h, ptr[bi, h, c]:ptr[bi, h, c + 1]]
                assert torch.equal(got, ref), (bi, h, c)
                assert end[bi, h, c] <= start[bi, h, c + 1]
                # each entry carries its key's four codes
                assert torch.equal(ic[bi, h, start[bi, h, c]:end[bi, h, c]], codes[bi, got.long(), h])


def test_decode_index_refuses_too_small_capacity():
    router = ssa.CodebookRouter(head_dim=64, route_dim=32, num_kv_heads=2, num_codebook=64, codes_per_key=4,
                                codes_per_query=8, top_k=16).to(DEV)
    cache = DecodeCache(router, 1, capacity=64, num_q_heads=4, dtype=torch.bfloat16, device=DEV)
    args = cache._args(64)
    small = L.SsaDecodeIndex.from_buffer_copy(cache.index)
    small.entry_capacity = 100
    ws = cache._workspace()
    rc = L.lib().ssa_decode_index_build(ctypes.byref(args), ctypes.byref(small), ws.data_ptr(), ws.numel(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 3 and b"slots" in L.lib().ssa_last_error()
