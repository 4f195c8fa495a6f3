"""Gradients of sparse exact attention (the backward kernel) on the GPU.

The reference differentiates its gather + einsum forward with autograd
(ssa/attention.py:93-113; tests/test_integration.py:32-49 checks that
gradients reach the q/k/v/o projections).  Here the kernel's dq, dk, dv are
compared with float64 autograd through a plain gather reference on the same
(rounded) inputs, for the per-head gather, causal masking with an offset,
duplicate indices and GQA groups; then gradient flow is checked through
SSAAttention and ToyTransformerBlock as the reference's tests do.
"""

import math

import numpy as np
import pytest
import torch

import ssa_b200 as ssa
from ssa_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _reference(q, k, v, idx, scale, causal, q_offset):
    """Gather attention in torch (per-head gather k[idx, h]), differentiable."""
    B, nq, hq, d = q.shape
    hkv = k.shape[2]
    g = hq // hkv
    bi = torch.arange(B, device=q.device)[:, None, None, None]
    hi = torch.arange(hkv, device=q.device)[None, None, :, None]
    ks = k[bi, idx, hi]                                           # [B, nq, hkv, kk, d]
    vs = v[bi, idx, hi]
    qg = q.reshape(B, nq, hkv, g, d)
    logits = torch.einsum("bnhgd,bnhtd->bnhgt", qg, ks) / scale
    if causal:
        pos = torch.arange(nq, device=q.device)[None, :, None, None] + q_offset
        logits = logits.masked_fill((idx > pos)[:, :, :, None, :], float("-inf"))
    p = torch.softmax(logits, dim=-1)
    return torch.einsum("bnhgt,bnhtd->bnhgd", p, vs).reshape(B, nq, hq, d)


def _case(seed, B, nq, n, hq, hkv, d, kk, dtype, causal, q_offset=0, dup=False):
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(rng.standard_normal((B, nq, hq, d)).astype(np.float32)).to(DEV, dtype)
    k = torch.from_numpy(rng.standard_normal((B, n, hkv, d)).astype(np.float32)).to(DEV, dtype)
    v = torch.from_numpy(rng.standard_normal((B, n, hkv, d)).astype(np.float32)).to(DEV, dtype)
    idx = rng.integers(0, n, size=(B, nq, hkv, kk))
    if causal:   # at least one valid key per row
        idx[..., 0] = rng.integers(0, q_offset + np.arange(nq) + 1)[None, :, None]
    if dup:
        idx[..., 1] = idx[..., 0]
    idx = torch.from_numpy(idx).to(DEV)
    go = torch.from_numpy(rng.standard_normal((B, nq, hq, d)).astype(np.float32)).to(DEV, dtype)
    return q, k, v, idx, go


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,nq,n,hq,hkv,d,kk,causal,q_offset,dup", [
    (1, 40, 40, 4, 1, 64, 16, True, 0, False),
    (2, 30, 70, 8, 2, 128, 24, True, 40, True),       # offset rows, duplicated slots
    (1, 25, 25, 28, 4, 128, 40, False, 0, False),     # g = 7, k > n
    (1, 20, 50, 16, 1, 32, 9, True, 30, False),       # g = 16, d = 32
])
def test_backward_matches_autograd_of_gather_reference(B, nq, n, hq, hkv, d, kk, causal, q_offset, dup, dtype):
    q, k, v, idx, go = _case(nq + d + kk, B, nq, n, hq, hkv, d, kk, dtype, causal, q_offset, dup)
    scale = math.sqrt(d)
    qr, kr, vr = (x.double().detach().requires_grad_() for x in (q, k, v))
    ref = _reference(qr, kr, vr, idx, scale, causal, q_offset)
    ref.backward(go.double())
    qq, kk_, vv = (x.detach().requires_grad_() for x in (q, k, v))
    out = ops.sparse_attn(qq, kk_, vv, idx, scale, causal, q_offset)
    out.backward(go)
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    for got, want, name in [(qq.grad, qr.grad, "dq"), (kk_.grad, kr.grad, "dk"), (vv.grad, vr.grad, "dv")]:
        assert got.dtype == dtype, name
        torch.testing.assert_close(got.double(), want, **tol, msg=name)


def test_backward_through_the_public_api_unbatched_int32():
    q, k, v, idx, go = _case(3, 1, 48, 48, 8, 2, 64, 12, torch.float32, True)
    scale = 2.5
    qr, kr, vr = (x.double().detach().requires_grad_() for x in (q, k, v))
    _reference(qr, kr, vr, idx, scale, True, 0).backward(go.double())
    qq, kk_, vv = (x[0].detach().requires_grad_() for x in (q, k, v))
    out = ssa.sparse_exact_attention(qq, kk_, vv, idx[0].to(torch.int32), scale=scale, is_causal=True)
    out.backward(go[0])
    for got, want in [(qq.grad, qr.grad[0]), (kk_.grad, kr.grad[0]), (vv.grad, vr.grad[0])]:
        torch.testing.assert_close(got.double(), want, rtol=1e-4, atol=1e-4)


def _module():
    torch.manual_seed(0)
    return ssa.SSAAttention(hidden_size=256, num_q_heads=4, num_kv_heads=1, head_dim=64, route_dim=16,
                            num_codebook=128, codes_per_key=4, codes_per_query=8, top_k=16).to(DEV)


def test_gradient_flow_reaches_projections_and_input():
    m = _module()
    x = torch.randn(2, 32, 256, device=DEV, requires_grad=True)
    m(x).sum().backward()
    for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
        grad = dict(m.named_parameters())[f"{name}.weight"].grad
        assert grad is not None and torch.isfinite(grad).all() and grad.abs().sum() > 0, name
    assert x.grad is not None and torch.isfinite(x.grad).all()


def test_toy_block_forward_backward_and_rope():
    torch.manual_seed(1)
    block = ssa.ToyTransformerBlock(hidden_size=256, num_q_heads=4, num_kv_heads=1, head_dim=64,
                                    top_k=16).to(DEV)
    x = torch.randn(2, 32, 256, device=DEV, requires_grad=True)
    out = block(x)
    assert out.shape == x.shape and torch.isfinite(out).all()
    out.sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    y = block(x.detach(), freqs=ssa.precompute_rope_freqs(64, 64).to(DEV))
    assert y.shape == x.shape


def test_module_smoke_behaviours():
    """The reference's module smoke tests: finite output, SSA vs dense of the
    same scale, variable lengths (k clamped), batch independence."""
    m = _module()
    with torch.no_grad():
        x = torch.randn(2, 32, 256, device=DEV)
        out_s, out_d = m(x), m(x, use_dense=True)
        assert torch.isfinite(out_s).all() and torch.isfinite(out_d).all()
        assert out_s.std() > 0 and out_d.std() > 0
        for n in (8, 16, 24, 32):
            assert m(torch.randn(1, n, 256, device=DEV)).shape == (1, n, 256)
        both = m(x)
        one_by_one = torch.cat([m(x[0:1]), m(x[1:2])])
        torch.testing.assert_close(both, one_by_one, rtol=0, atol=1e-6)
    with pytest.raises(NotImplementedError):
        m.compute_auxiliary_loss(x)
