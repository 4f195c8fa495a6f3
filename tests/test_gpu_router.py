"""End-to-end router and module parity on the GPU.

* the reference's own fixtures (codes, well-defined top-k rows, module
  output) reproduced through the public API;
* code overlap and final candidate-set overlap >= 99.9% against the float64
  oracle on a planted-cluster config-3 slice (bf16);
* k = n reproduces dense causal attention (config 2, fp32 and bf16).
"""

import math
import os

import numpy as np
import pytest
import torch

import ssa_b200 as ssa
from oracle import ssa_oracle as O
from ssa_b200 import workloads as W
from _tol import assert_output_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _router_from(z, dims):
    n, h_q, h_kv, d, d_s, n_c, a, b, k = (int(x) for x in dims)
    r = ssa.CodebookRouter(head_dim=d, route_dim=d_s, num_kv_heads=h_kv, num_codebook=n_c,
                           codes_per_key=b, codes_per_query=a, top_k=k).to(DEV)
    with torch.no_grad():
        r.W_qr.weight.copy_(torch.from_numpy(z["w_qr"]))
        r.W_kr.weight.copy_(torch.from_numpy(z["w_kr"]))
        r.codebook.copy_(torch.from_numpy(z["codebook"]))
    return r


def test_router_reproduces_reference_fixture():
    z = np.load(os.path.join(GOLD, "stage1.npz"))
    r = _router_from(z, z["dims"])
    q = torch.from_numpy(z["q"]).to(DEV)
    k = torch.from_numpy(z["k"]).to(DEV)
    idx, q_codes, k_codes, _ = r.route(q[None], k[None], causal=True)
    np.testing.assert_array_equal(q_codes[0].cpu().numpy(), z["top_q_codes"])
    np.testing.assert_array_equal(k_codes[0].cpu().numpy(), z["k_code_assign"])
    wd = z["well_defined"]
    np.testing.assert_array_equal(idx[0].cpu().numpy()[wd], z["indices"][wd])
    # public forward(): causal mask form and README causal= form agree
    a = r(q, k, causal_mask=ssa.build_causal_mask(q.shape[0], device=DEV))
    b2 = r(q, k, causal=True)
    assert a.dtype == torch.int64 and torch.equal(a, b2) and torch.equal(a, idx[0])
    ca = r.get_code_assignment(k)
    np.testing.assert_array_equal(ca.cpu().numpy(), z["k_code_assign"])


def test_module_reproduces_reference_fixture():
    z = np.load(os.path.join(GOLD, "module.npz"))
    hs, h_q, h_kv, d, n, d_s, n_c, b, a, k = (int(x) for x in z["dims"])
    m = ssa.SSAAttention(hidden_size=hs, num_q_heads=h_q, num_kv_heads=h_kv, head_dim=d, route_dim=d_s,
                         num_codebook=n_c, codes_per_key=b, codes_per_query=a, top_k=k)
    sd = {kk[3:].replace("__", "."): torch.from_numpy(z[kk]) for kk in z.files if kk.startswith("sd_")}
    m.load_state_dict(sd)
    m = m.to(DEV)
    with torch.no_grad():
        y = m(torch.from_numpy(z["x"]).to(DEV), freqs=torch.from_numpy(z["freqs"]).to(DEV))
    rows = z["well_defined_rows"]
    np.testing.assert_allclose(y[0].cpu().numpy()[rows], z["y"][0][rows], rtol=1e-4, atol=1e-5)
    # every row (including filler rows) against the oracle's canonical module
    w = {kk: v.numpy() for kk, v in sd.items()}
    y_or, _ = O.module_forward(z["x"], w, h_q, h_kv, d, n_c, a, b, k, freqs=z["freqs"])
    np.testing.assert_allclose(y[0].cpu().numpy(), y_or[0], rtol=1e-4, atol=1e-5)


def _overlap(a, b):
    """Mean |set(a_row) & set(b_row)| / k over rows of [..., k] index arrays."""
    a = np.sort(a.reshape(-1, a.shape[-1]), axis=1)
    b = np.sort(b.reshape(-1, b.shape[-1]), axis=1)
    hits = 0
    for x, y in zip(a, b):
        hits += np.intersect1d(x, y, assume_unique=False).size
    return hits / a.size


def test_config3_slice_overlap_bf16():
    shape = W.Shape(n=4096, h_q=32, h_kv=8, d=128, d_s=32, n_codes=4096, a=16, b=4, top_k=256)
    t = W.make_inputs(shape, seed=3, dtype=torch.bfloat16)
    r = ssa.CodebookRouter(head_dim=128, route_dim=32, num_kv_heads=8, num_codebook=4096,
                           codes_per_key=4, codes_per_query=16, top_k=256).to(DEV)
    with torch.no_grad():
        r.W_qr.weight.copy_(t["w_qr"])
        r.W_kr.weight.copy_(t["w_kr"])
        r.codebook.copy_(t["codebook"])
    idx, q_codes, k_codes, counts = r.route(t["q"], t["k"], causal=True)
    qn = t["q"][0].double().cpu().numpy()
    kn = t["k"][0].double().cpu().numpy()
    oq, ok = O.route_codes(qn, kn, t["w_qr"].cpu().numpy(), t["w_kr"].cpu().numpy(),
                           t["codebook"].cpu().numpy(), 16, 4)
    q_same = (np.sort(q_codes[0].cpu().numpy(), -1) == np.sort(oq, -1)).all(-1).mean()
    k_same = (np.sort(k_codes[0].cpu().numpy(), -1) == np.sort(ok, -1)).all(-1).mean()
    assert q_same >= 0.999 and k_same >= 0.999, (q_same, k_same)
    ref = O.select_topk_index(qn, kn, oq, ok, 4096, 256, causal=True)
    ov = _overlap(idx[0].cpu().numpy(), ref)
    assert ov >= 0.999, ov
    # stage 3 on the GPU's own indices against the oracle on the same indices
    v = t["v"]
    out = ssa.sparse_exact_attention(t["q"][0], t["k"][0], v[0], idx[0], is_causal=True)
    ref_out = O.sparse_attention(qn, kn, v[0].double().cpu().numpy(), idx[0].cpu().numpy(), causal=True)
    assert_output_close(out, ref_out, torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_k_equals_n_reproduces_dense(dtype):
    shape = W.CONFIG2
    t = W.make_inputs(shape, seed=2, dtype=dtype, planted=False)
    r = ssa.CodebookRouter(head_dim=64, route_dim=32, num_kv_heads=2, num_codebook=1024,
                           codes_per_key=4, codes_per_query=16, top_k=4096).to(DEV)
    q, k, v = t["q"][0], t["k"][0], t["v"][0]
    idx = r(q, k, causal=True)
    srt = torch.sort(idx, dim=-1).values
    assert torch.equal(srt, torch.arange(4096, device=DEV).expand_as(srt))
    out = ssa.sparse_exact_attention(q, k, v, idx, is_causal=True)
    qd, kd, vd = q.double(), k.double(), v.double()
    dense = ssa.dense_attention(qd, kd, vd, causal_mask=ssa.build_causal_mask(4096, device=DEV))
    assert_output_close(out, dense, dtype)


@pytest.mark.parametrize("d_s,n_codes,shared_cb,temp,dtype", [
    (32, 512, False, 1.0, torch.float32),
    (16, 1024, True, 0.7, torch.bfloat16),
    (32, 4096, False, 1.0, torch.bfloat16),
])
def test_tensor_core_code_selection_matches_oracle(d_s, n_codes, shared_cb, temp, dtype):
    """Shapes that take the tcgen05 scoring path (d_s 16/32, N_c % 256 == 0);
    row counts are not multiples of the 128-row tile; batch of 2."""
    B, n, h_q, h_kv, d, a, b = 2, 1000, 8, 2, 64, 16, 4
    g = torch.Generator().manual_seed(n_codes + d_s)
    q = torch.randn(B, n, h_q, d, generator=g).to(DEV, dtype)
    k = torch.randn(B, n, h_kv, d, generator=g).to(DEV, dtype)
    r = ssa.CodebookRouter(head_dim=d, route_dim=d_s, num_kv_heads=h_kv, num_codebook=n_codes,
                           codes_per_key=b, codes_per_query=a, top_k=32, temperature=temp).to(DEV)
    if shared_cb:
        r.codebook = torch.nn.Parameter(torch.randn(n_codes, d_s, generator=g).to(DEV) / d_s ** 0.5)
    _, q_codes, k_codes, _ = r.route(q, k, causal=True)
    w = lambda p: p.detach().double().cpu().numpy()
    for bi in range(B):
        oq, ok = O.route_codes(q[bi].double().cpu().numpy(), k[bi].double().cpu().numpy(), w(r.W_qr.weight),
                               w(r.W_kr.weight), w(r.codebook), a, b, temperature=temp)
        q_rows = (np.sort(q_codes[bi].cpu().numpy(), -1) == np.sort(oq, -1)).all(-1).mean()
        k_rows = (np.sort(k_codes[bi].cpu().numpy(), -1) == np.sort(ok, -1)).all(-1).mean()
        assert q_rows >= 0.999 and k_rows >= 0.999, (q_rows, k_rows)
    kc = r.get_code_assignment(k)
    assert torch.equal(kc.int(), k_codes)


def test_batched_module_matches_per_sequence_calls():
    m = ssa.SSAAttention(hidden_size=256, num_q_heads=4, num_kv_heads=1, head_dim=64, route_dim=16,
                         num_codebook=128, codes_per_key=4, codes_per_query=8, top_k=16).to(DEV)
    x = torch.randn(2, 32, 256, device=DEV)
    with torch.no_grad():
        y = m(x)
        y0, y1 = m(x[:1]), m(x[1:])
    assert torch.allclose(y, torch.cat([y0, y1]), atol=1e-6)
    with torch.no_grad():
        yd = m(x, use_dense=True)
    assert torch.isfinite(yd).all() and torch.isfinite(y).all()


def test_router_deterministic_and_variable_lengths():
    r = ssa.CodebookRouter(head_dim=64, route_dim=16, num_kv_heads=2, num_codebook=128, codes_per_key=4,
                           codes_per_query=8, top_k=16).to(DEV)
    for n in (1, 8, 16, 24, 33, 1000):
        q = torch.randn(n, 8, 64, device=DEV)
        k = torch.randn(n, 2, 64, device=DEV)
        a = r(q, k, causal=True)
        b = r(q, k, causal=True)
        assert a.shape == (n, 2, 16) and torch.equal(a, b)
        assert int(a.min()) >= 0 and int(a.max()) < n


def _random_router(n_c=1024, d=128, d_s=32, h_kv=2, a=8, b=4, k=64, seed=3):
    torch.manual_seed(seed)
    return ssa.CodebookRouter(head_dim=d, route_dim=d_s, num_kv_heads=h_kv, num_codebook=n_c,
                              codes_per_key=b, codes_per_query=a, top_k=k).to(DEV)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_route_with_key_codes_matches_route_on_query_shards(dtype):
    r = _random_router()
    g = torch.Generator(device="cpu").manual_seed(5)
    n = 3000
    q = torch.randn((2, n, 8, 128), generator=g).to(DEV, dtype)
    k = torch.randn((2, n, 2, 128), generator=g).to(DEV, dtype)
    full, _, k_codes, _ = r.route(q, k, causal=True)
    codes = r.key_codes(k)
    assert torch.equal(codes, k_codes)
    for start, length in [(0, 700), (700, 1100), (1800, 1200), (2999, 1)]:
        got = r.route_with_key_codes(q[:, start:start + length], k, codes, causal=True, q_offset=start)
        assert torch.equal(got, full[:, start:start + length]), (start, length)


def test_route_with_key_codes_flags_codes_outside_the_codebook():
    r = _random_router(n_c=512)
    q = torch.randn((1, 600, 8, 128), device=DEV, dtype=torch.bfloat16)
    k = torch.randn((1, 600, 2, 128), device=DEV, dtype=torch.bfloat16)
    codes = r.key_codes(k)
    for bad in (512, -1, 1 << 20):
        c = codes.clone()
        c[0, 17, 1, 2] = bad
        with pytest.raises(ValueError, match="outside"):
            r.route_with_key_codes(q, k, c, causal=True)
            ssa.check_errors()
    # the device word is clear again on valid codes
    r.route_with_key_codes(q, k, codes, causal=True)
    torch.cuda.synchronize()


def test_route_with_key_codes_refuses_unaligned_codes():
    from ssa_b200._lib import SSAError
    r = _random_router(n_c=512)
    q = torch.randn((1, 64, 8, 128), device=DEV, dtype=torch.bfloat16)
    k = torch.randn((1, 64, 2, 128), device=DEV, dtype=torch.bfloat16)
    codes = r.key_codes(k)
    buf = torch.empty(codes.numel() + 1, dtype=torch.int32, device=DEV)
    shifted = buf[1:].view(codes.shape)                      # 4 bytes past a 16-byte boundary
    shifted.copy_(codes)
    with pytest.raises(SSAError, match="aligned"):
        r.route_with_key_codes(q, k, shifted, causal=True)


def test_route_with_index_matches_route_on_query_shards():
    r = _random_router()
    g = torch.Generator(device="cpu").manual_seed(6)
    n = 2500
    q = torch.randn((2, n, 8, 128), generator=g).to(DEV, torch.bfloat16)
    k = torch.randn((2, n, 2, 128), generator=g).to(DEV, torch.bfloat16)
    full, _, _, _ = r.route(q, k, causal=True)
    codes = r.key_codes(k)
    index = r.key_index(codes)
    for start, length in [(0, 900), (900, 1600), (2499, 1)]:
        got = r.route_with_index(q[:, start:start + length], k, codes, index, causal=True, q_offset=start)
        assert torch.equal(got, full[:, start:start + length]), (start, length)


def test_route_with_index_refuses_a_corrupt_index():
    r = _random_router(n_c=512)
    q = torch.randn((1, 700, 8, 128), device=DEV, dtype=torch.bfloat16)
    k = torch.randn((1, 700, 2, 128), device=DEV, dtype=torch.bfloat16)
    codes = r.key_codes(k)
    ptr, keys = r.key_index(codes)
    good = r.route_with_index(q, k, codes, (ptr, keys), causal=True)
    bad_key = keys.clone()
    bad_key[0, 1, 33] = 700
    bad_order = ptr.clone()
    bad_order[0, 0, 100] = bad_order[0, 0, 102] + 1
    bad_end = ptr.clone()
    bad_end[0, 1, -1] = 700 * 4 + 1
    for index in [(ptr, bad_key), (bad_order, keys), (bad_end, keys)]:
        with pytest.raises(ValueError, match="index"):
            r.route_with_index(q, k, codes, index, causal=True)
            ssa.check_errors()
    # a valid index still gives the same result afterwards
    assert torch.equal(r.route_with_index(q, k, codes, (ptr, keys), causal=True), good)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_segment_calls_match_the_full_route_and_attention(dtype):
    """A rank's zig-zag blocks routed and attended in one call each (query
    segments) give exactly the full sequence's rows."""
    from ssa_b200 import ops, shard

    r = _random_router()
    g = torch.Generator(device="cpu").manual_seed(9)
    n = 3072
    q = torch.randn((2, n, 8, 128), generator=g).to(DEV, dtype)
    k = torch.randn((2, n, 2, 128), generator=g).to(DEV, dtype)
    v = torch.randn((2, n, 2, 128), generator=g).to(DEV, dtype)
    full, _, codes, _ = r.route(q, k, causal=True, index_dtype=torch.int32)
    out_full = ops.sparse_attn(q, k, v, full, 128 ** 0.5, True, 0)
    index = r.key_index(codes)
    for world, folds, rank in [(2, 1, 0), (3, 2, 2), (4, 1, 3)]:
        blocks = shard.zigzag_blocks(n, world, rank, folds)
        ql = shard.local_rows(q, world, rank, folds=folds)
        idx = ops.route_with_index_segments(ql, k, codes, index[0], index[1], r.W_qr.weight.detach(),
                                            r.W_kr.weight.detach(), r.codebook.detach(), r.codes_per_query,
                                            r.top_k, True, 1.0, blocks)
        assert torch.equal(idx, shard.local_rows(full, world, rank, folds=folds)), (world, folds, rank)
        # the same call split in two: query codes first (no keys), then stage 2
        qc = ops.query_codes(ql, r.W_qr.weight.detach(), r.codebook.detach(), r.codes_per_query, 2)
        idx2 = ops.select_candidates_segments(ql, k, qc, codes, index[0], index[1], r.top_k, True, blocks)
        assert torch.equal(idx2, idx), (world, folds, rank)
        out = ops.sparse_attn_segments(ql, k, v, idx, 128 ** 0.5, True, blocks)
        assert torch.equal(out, shard.local_rows(out_full, world, rank, folds=folds)), (world, folds, rank)
    ssa.check_errors()
