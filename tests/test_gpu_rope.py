"""RoPE fused into the routing projection (``ssa_route_rope``) against the
unfused path: the PyTorch rotate-half expression of the Qwen2 path
(``x * cos + cat(-x2, x1) * sin``, ``training/train_qwen.py:134-135``) followed
by ``CodebookRouter.route``.  The rotated rows must be bit-identical to the
PyTorch expression and the indices identical to routing the rotated rows."""

import pytest
import torch

import ssa_b200 as ssa

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tables(positions, d, theta, dtype, shift=0):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, device=DEV, dtype=torch.float32) / d))
    ang = (torch.arange(positions, device=DEV, dtype=torch.float32) + shift)[:, None] * inv[None, :]
    emb = torch.cat([ang, ang], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rope(x, cos, sin):
    """x [B, n, h, d]; cos / sin broadcastable to it."""
    h = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., h:], x[..., :h]], dim=-1) * sin


def _router(d, h_kv, n_codes, top_k):
    torch.manual_seed(0)
    return ssa.CodebookRouter(head_dim=d, route_dim=32, num_kv_heads=h_kv, num_codebook=n_codes,
                              codes_per_key=4, codes_per_query=16, top_k=top_k).to(DEV)


def test_route_rope_matches_rope_then_route_bf16_per_sequence_tables():
    B, n, h_q, h_kv, d = 2, 1000, 8, 2, 128
    g = torch.Generator(device=DEV).manual_seed(1)
    q = torch.randn(B, n, h_q, d, generator=g, device=DEV).bfloat16()
    k = torch.randn(B, n, h_kv, d, generator=g, device=DEV).bfloat16()
    c0, s0 = _tables(n, d, 1e6, torch.bfloat16)
    c1, s1 = _tables(n, d, 1e6, torch.bfloat16, shift=37)         # second sequence starts at position 37
    cos, sin = torch.stack([c0, c1]), torch.stack([s0, s1])       # [B, n, d]
    r = _router(d, h_kv, 512, 32)
    q_ref, k_ref = _rope(q, cos[:, :, None], sin[:, :, None]), _rope(k, cos[:, :, None], sin[:, :, None])
    idx_ref = r.route(q_ref, k_ref, causal=True)[0]
    idx, q_rot, k_rot = r.route_rope(q, k, cos, sin, causal=True)
    assert torch.equal(q_rot, q_ref) and torch.equal(k_rot, k_ref)
    assert torch.equal(idx, idx_ref)


def test_route_rope_query_shard_f16_head_dim_64_shared_table():
    B, n, h_q, h_kv, d, start, rows = 1, 777, 12, 4, 64, 300, 200
    g = torch.Generator(device=DEV).manual_seed(2)
    q = torch.randn(B, rows, h_q, d, generator=g, device=DEV).half()
    k = torch.randn(B, n, h_kv, d, generator=g, device=DEV).half()
    cos, sin = _tables(n, d, 1e4, torch.float16)                  # [n, d], shared by the batch
    r = _router(d, h_kv, 1024, 24)
    q_ref = _rope(q, cos[start:start + rows, None], sin[start:start + rows, None])
    k_ref = _rope(k, cos[:, None], sin[:, None])
    idx_ref = r.route(q_ref, k_ref, causal=True, q_offset=start)[0]
    idx, q_rot, k_rot = r.route_rope(q, k, cos, sin, causal=True, q_offset=start)
    assert torch.equal(q_rot, q_ref) and torch.equal(k_rot, k_ref)
    assert torch.equal(idx, idx_ref)


def test_route_rope_on_head_major_views_then_attention():
    """q/k as [B, n, h, d] views of [B, h, n, d] memory (the layout of the
    Qwen2 projections after .transpose(1, 2)); the rotated rows feed the
    sparse attention exactly as the unfused ones."""
    B, n, h_q, h_kv, d = 1, 513, 7, 1, 128
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(B, h_q, n, d, generator=g, device=DEV).bfloat16().transpose(1, 2)
    k = torch.randn(B, h_kv, n, d, generator=g, device=DEV).bfloat16().transpose(1, 2)
    v = torch.randn(B, n, h_kv, d, generator=g, device=DEV).bfloat16()
    cos, sin = _tables(n, d, 1e6, torch.bfloat16)
    cos4, sin4 = cos[None, :, None], sin[None, :, None]          # [1, n, 1, d] broadcast form
    r = _router(d, h_kv, 512, 64)
    q_ref, k_ref = _rope(q, cos4, sin4), _rope(k, cos4, sin4)
    idx_ref = r.route(q_ref, k_ref, causal=True)[0]
    idx, q_rot, k_rot = r.route_rope(q, k, cos4, sin4, causal=True)
    assert torch.equal(q_rot, q_ref) and torch.equal(k_rot, k_ref) and torch.equal(idx, idx_ref)
    out = ssa.sparse_exact_attention(q_rot[0], k_rot[0], v[0], idx[0], is_causal=True)
    ref = ssa.sparse_exact_attention(q_ref[0].contiguous(), k_ref[0].contiguous(), v[0], idx_ref[0],
                                     is_causal=True)
    assert torch.equal(out, ref)


def test_route_rope_rejects_fp32_and_short_tables():
    r = _router(128, 2, 512, 32)
    q = torch.randn(1, 64, 4, 128, device=DEV)
    k = torch.randn(1, 64, 2, 128, device=DEV)
    cos, sin = _tables(64, 128, 1e4, torch.float32)
    with pytest.raises(RuntimeError):
        r.route_rope(q, k, cos, sin)                               # fp32: SSA_ERR_UNSUPPORTED
    cos, sin = _tables(32, 128, 1e4, torch.bfloat16)
    with pytest.raises(ValueError):
        r.route_rope(q.bfloat16(), k.bfloat16(), cos, sin)         # 32 positions for 64 rows
