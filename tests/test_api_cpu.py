"""Host-side behaviour of the drop-in ``ssa`` API (no GPU needed)."""

import os

import numpy as np
import pytest
import torch

import ssa_b200 as ssa
from oracle import ssa_oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_public_names_match_reference_package():
    for name in ["CodebookRouter", "sparse_exact_attention", "dense_attention", "SSAAttention",
                 "ToyTransformerBlock", "apply_rope", "precompute_rope_freqs", "build_causal_mask",
                 "expand_kv_for_gqa"]:
        assert name in ssa.__all__ and hasattr(ssa, name)


def test_router_code_and_readme_spellings_agree():
    r1 = ssa.CodebookRouter(head_dim=64, route_dim=32, num_kv_heads=2, num_codebook=256,
                            codes_per_key=4, codes_per_query=16, top_k=32)
    r2 = ssa.CodebookRouter(d=64, d_s=32, n_c=256, b=4, a=16, k=32, num_kv_heads=2)
    for attr in ["head_dim", "route_dim", "num_codebook", "codes_per_key", "codes_per_query", "top_k"]:
        assert getattr(r1, attr) == getattr(r2, attr)
    with pytest.raises(TypeError):
        ssa.CodebookRouter(bogus=1)


def test_state_dict_keys_match_reference():
    z = np.load(os.path.join(GOLD, "module.npz"))
    ref_keys = sorted(k[3:].replace("__", ".") for k in z.files if k.startswith("sd_"))
    hs, h_q, h_kv, d, n, d_s, n_c, b, a, k = z["dims"]
    m = ssa.SSAAttention(hidden_size=int(hs), num_q_heads=int(h_q), num_kv_heads=int(h_kv),
                         head_dim=int(d), route_dim=int(d_s), num_codebook=int(n_c),
                         codes_per_key=int(b), codes_per_query=int(a), top_k=int(k))
    assert sorted(m.state_dict().keys()) == ref_keys
    sd = {kk: torch.from_numpy(z["sd_" + kk.replace(".", "__")]) for kk in ref_keys}
    m.load_state_dict(sd)      # reference checkpoints load unchanged


def test_readme_module_spelling():
    m = ssa.SSAAttention(d_model=128, h_q=4, h_kv=2, d_head=32, d_s=16, n_c=64, b=4, a=8, k=16,
                         causal=True)
    assert m.num_q_heads == 4 and m.router.num_codebook == 64 and m.top_k == 16


def test_cpu_tensors_raise_no_fallback():
    r = ssa.CodebookRouter(head_dim=16, route_dim=8, num_kv_heads=1, num_codebook=16,
                           codes_per_key=2, codes_per_query=4, top_k=4)
    q = torch.randn(8, 2, 16)
    k = torch.randn(8, 1, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        r(q, k, causal_mask=ssa.build_causal_mask(8))
    with pytest.raises(RuntimeError, match="CUDA"):
        ssa.sparse_exact_attention(q, k, k, torch.zeros(8, 1, 4, dtype=torch.long))


def test_gumbel_mode_is_not_provided():
    r = ssa.CodebookRouter(head_dim=16, route_dim=8, num_kv_heads=1, num_codebook=16,
                           codes_per_key=2, codes_per_query=4, top_k=4)
    with pytest.raises(NotImplementedError):
        r(torch.randn(8, 2, 16), torch.randn(8, 1, 16), hard=False)


def test_only_lower_triangular_masks_are_accepted():
    r = ssa.CodebookRouter(head_dim=16, route_dim=8, num_kv_heads=1, num_codebook=16,
                           codes_per_key=2, codes_per_query=4, top_k=4)
    bad = torch.ones(8, 8, dtype=torch.bool)
    with pytest.raises(ValueError):
        r(torch.randn(8, 2, 16), torch.randn(8, 1, 16), causal_mask=bad)
    tril = torch.ones(8, 8, dtype=torch.bool).tril()      # untagged but lower-triangular
    assert r._causal_flag(tril, None) is True
    assert r._causal_flag(None, None) is False
    assert r._causal_flag(None, True) is True


def test_rope_matches_reference_restatement():
    z = np.load(os.path.join(GOLD, "module.npz"))
    freqs = torch.from_numpy(z["freqs"])
    x = torch.randn(10, 4, 32, dtype=torch.float64)
    ours = ssa.apply_rope(x, freqs[:10]).numpy()
    np.testing.assert_allclose(ours, O.rope_reference(x.numpy(), z["freqs"][:10]), atol=1e-12)
    # reference helper test: (t, t + d/4) pair norms are preserved
    y = ssa.apply_rope(x[:, 0], ssa.precompute_rope_freqs(32, 20))
    q4 = 8
    np.testing.assert_allclose((x[:, 0, :q4] ** 2 + x[:, 0, q4:2 * q4] ** 2).numpy(),
                               (y[:, :q4] ** 2 + y[:, q4:2 * q4] ** 2).numpy(), atol=1e-10)


def test_dense_attention_torch_path_matches_oracle():
    z = np.load(os.path.join(GOLD, "dense.npz"))
    out = ssa.dense_attention(*(torch.from_numpy(z[t]) for t in "qkv"),
                              causal_mask=ssa.build_causal_mask(48))
    np.testing.assert_allclose(out.numpy(), z["out"], rtol=1e-5, atol=1e-5)


def test_expand_kv_and_validate_indices():
    # the reference's own outputs (tests/golden/make_golden.py): head tiling,
    # query head j -> KV head j % h_kv
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "gqa_expand.npz"))
    for name in ("u", "b", "one"):
        kv = torch.from_numpy(z[f"kv_{name}"])
        e = ssa.expand_kv_for_gqa(kv, int(z[f"hq_{name}"]), kv.shape[-2])
        assert torch.equal(e, torch.from_numpy(z[f"out_{name}"])), name
    kv = torch.randn(5, 2, 3)
    e = ssa.expand_kv_for_gqa(kv, 6, 2)
    assert [torch.equal(e[:, j], kv[:, j % 2]) for j in range(6)] == [True] * 6
    ssa.validate_indices(torch.zeros(4, 1, 3, dtype=torch.long), 4, 3)
    with pytest.raises(ValueError):
        ssa.validate_indices(torch.full((4, 1, 3), 4), 4, 3)
