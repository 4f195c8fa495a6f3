"""The two stage-2 re-score paths give the same indices bit for bit.

The bucket-major path (rescore_bucket.cu: queries and keys of one code meet
in a tile, scores go through per-query segments) and the walking kernel
(rescore_mma.cu: each query walks its buckets) compute every unit's scores
with the same tensor-core fragments and share the selection code, so their
outputs, candidate counts included, must be identical -- whichever units the
bucket path hands to the walking kernel for lack of room.  Checked on bf16
and fp16, d 64 and 128, k up to 512, causal and not, with codebooks small
enough that many queries hold more candidates than a shared-memory batch
(the path that selects straight from the segment).  The oracle checks of the
other GPU tests run through the bucket path, which is the default.
"""

import os

import pytest
import torch

import ssa_b200 as ssa

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _route(q, k, r, causal, env=None):
    old = {x: os.environ.get(x) for x in ("SSA_RESCORE", "SSA_RESCORE_UNIT_ROOM")}
    try:
        for x in old:
            os.environ.pop(x, None)
        os.environ.update(env or {})
        idx, qc, kc, counts = r.route(q, k, causal=causal, index_dtype=torch.int32)
        torch.cuda.synchronize()
        ssa.check_errors()
        return idx, counts
    finally:
        for x, v in old.items():
            if v is None:
                os.environ.pop(x, None)
            else:
                os.environ[x] = v


def _problem(n, h_q, h_kv, d, n_c, a, k, dtype, seed, batch=2):
    g = torch.Generator(device="cpu").manual_seed(seed)
    r = ssa.CodebookRouter(head_dim=d, route_dim=32, num_kv_heads=h_kv, num_codebook=n_c, codes_per_key=4,
                           codes_per_query=a, top_k=k).to(DEV)
    with torch.no_grad():
        r.W_qr.weight.copy_(torch.randn(32, d, generator=g))
        r.W_kr.weight.copy_(torch.randn(32, d, generator=g))
        r.codebook.copy_(torch.randn(h_kv, n_c, 32, generator=g))
    q = torch.randn((batch, n, h_q, d), generator=g).to(DEV, dtype)
    k_ = torch.randn((batch, n, h_kv, d), generator=g).to(DEV, dtype)
    return r, q, k_


CASES = [
    # n, h_q, h_kv, d, n_codes, a, k, dtype, causal
    (4096, 8, 2, 128, 1024, 16, 256, torch.bfloat16, True),
    (4096, 8, 2, 128, 1024, 16, 512, torch.bfloat16, True),
    (2048, 8, 2, 64, 512, 16, 128, torch.float16, True),
    (2048, 14, 2, 128, 256, 16, 256, torch.bfloat16, True),       # g = 7, ~500 candidates a query
    (1024, 8, 2, 128, 256, 8, 64, torch.bfloat16, False),
    (4096, 4, 4, 64, 256, 32, 512, torch.float16, False),         # a = 32, > 1024 candidates
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"n{c[0]}-g{c[1] // c[2]}-d{c[3]}-nc{c[4]}-a{c[5]}-k{c[6]}-"
                                                     f"{str(c[7]).split('.')[-1]}-{'causal' if c[8] else 'full'}")
def test_bucket_path_matches_walking_kernel(case):
    n, h_q, h_kv, d, n_c, a, k, dtype, causal = case
    r, q, kk = _problem(n, h_q, h_kv, d, n_c, a, k, dtype, seed=n + d + a)
    walk, walk_counts = _route(q, kk, r, causal, {"SSA_RESCORE": "walk"})
    bucket, bucket_counts = _route(q, kk, r, causal)
    assert torch.equal(bucket_counts, walk_counts)
    assert torch.equal(bucket, walk)
    # most units overflow the buffer: the walking kernel finishes them
    part, part_counts = _route(q, kk, r, causal, {"SSA_RESCORE_UNIT_ROOM": "96"})
    assert torch.equal(part_counts, walk_counts) and torch.equal(part, walk)


def test_bucket_path_selects_from_segments_larger_than_shared_memory():
    """A 64-code codebook gives most queries of a 2048-key causal head far more
    candidates than the 512 keys a warp holds in shared memory."""
    r, q, kk = _problem(2048, 8, 2, 128, 64, 16, 256, torch.bfloat16, seed=7)
    walk, wc = _route(q, kk, r, True, {"SSA_RESCORE": "walk"})
    bucket, bc = _route(q, kk, r, True)
    assert (bc > 512).float().mean().item() > 0.25
    assert torch.equal(bc, wc) and torch.equal(bucket, walk)
