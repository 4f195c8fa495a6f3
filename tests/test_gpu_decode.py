"""Token-by-token decoding (ssa_b200.decode.DecodeCache) against the
full-sequence forward.

Every per-row computation of a decode step (the key's codes, the query's
codes, candidates, re-score, top-k, attention) is the one the full forward
does for that row, so from position top_k - 1 on (where the full forward's
filler keys are all in the past) the outputs are identical.
"""

import math

import pytest
import torch

import ssa_b200 as ssa
from ssa_b200.decode import DecodeCache

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_steps_match_the_full_forward(dtype):
    torch.manual_seed(0)
    B, n, h_q, h_kv, d, top_k = 2, 96, 8, 2, 64, 16
    router = ssa.CodebookRouter(head_dim=d, route_dim=32, num_kv_heads=h_kv, num_codebook=256,
                                codes_per_key=4, codes_per_query=8, top_k=top_k).to(DEV)
    g = torch.Generator(device="cpu").manual_seed(1)
    q = torch.randn((B, n, h_q, d), generator=g).to(DEV, dtype)
    k = torch.randn((B, n, h_kv, d), generator=g).to(DEV, dtype)
    v = torch.randn((B, n, h_kv, d), generator=g).to(DEV, dtype)
    idx = router.route(q, k, causal=True)[0]
    full = ssa.sparse_exact_attention(q, k, v, idx, is_causal=True)

    cache = DecodeCache(router, B, capacity=128, num_q_heads=h_q, dtype=dtype, device=DEV)
    p0 = 20
    cache.append(k[:, :p0], v[:, :p0])
    assert torch.equal(cache.codes[:, :p0], router.key_codes(k[:, :p0]))
    for p in range(p0, n):
        out = cache.step(q[:, p:p + 1], k[:, p:p + 1], v[:, p:p + 1])
        assert out.shape == (B, 1, h_q, d)
        assert torch.equal(out, full[:, p:p + 1]), p
    assert cache.n == n
    with pytest.raises(ValueError, match="full"):
        cache.append(torch.empty((B, 40, h_kv, d), device=DEV, dtype=dtype),
                     torch.empty((B, 40, h_kv, d), device=DEV, dtype=dtype))
