"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run where the reference implementation's source tree is available, with
``SSA_REFERENCE_PATH`` set to its root (the directory holding the ``ssa``
package):

    SSA_REFERENCE_PATH=<reference checkout> python tests/golden/make_golden.py

Each fixture stores seeded inputs together with the outputs of the
*unmodified* reference code (chenxingqiang/SSA, pure PyTorch, fp32, CPU):

* ``stage1.npz``    -- routing: ``q_code_scores``, ``k_code_assign`` and
  ``top_q_codes`` captured at ``CodebookRouter._select_candidates``
  (ssa/router.py:145-147), the candidate mask from
  ``_build_candidate_mask`` (ssa/router.py:216-259), and the final indices
  plus a per-row flag saying where the reference's top-k is well defined
  (at least ``min(k,n)`` finite scores, so no ``-inf`` filler).
* ``stage3_h1.npz`` -- ``sparse_exact_attention`` (ssa/attention.py:12-115)
  with ``num_kv_heads = 1``, where its flattened gather is correct.
* ``stage3_h2.npz`` -- the same at ``num_kv_heads = 2``: the raw output, which
  follows the reference's ``h*seq_len`` row mapping (ssa/attention.py:76-91).
* ``dense.npz``     -- ``dense_attention`` with a causal mask
  (ssa/attention.py:118-158).
* ``module.npz``    -- ``SSAAttention.forward`` (ssa/ssa_layer.py:68-138) with
  RoPE, ``num_kv_heads = 1``; the RoPE'd ``q``/``k`` handed to the router
  (captured at ssa/ssa_layer.py:129) and the rows whose selection is well
  defined.
* ``gqa_expand.npz`` -- ``expand_kv_for_gqa`` (ssa/utils.py:89-106) on
  unbatched and batched inputs for several group sizes.

``--only gqa_expand`` writes that one fixture and leaves the others as they are.

The reference directory is read-only, so bytecode writing is disabled.
"""

from __future__ import annotations

import os
import sys

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("SSA_REFERENCE_PATH", "")


def _import_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "ssa")):
        raise SystemExit("set SSA_REFERENCE_PATH to the reference checkout (the directory holding `ssa/`)")
    sys.path.insert(0, REF)
    import ssa  # noqa: F401  (the reference package)
    assert os.path.realpath(os.path.dirname(ssa.__file__)).startswith(os.path.realpath(REF))
    return ssa


def gqa_expand(ssa):
    import numpy as np
    import torch

    torch.manual_seed(31)
    out = {}
    for name, shape, h_q in (("u", (5, 2, 3), 6), ("b", (2, 4, 3, 8), 12), ("one", (3, 1, 4), 4)):
        kv = torch.randn(*shape)
        out[f"kv_{name}"] = kv.numpy()
        out[f"out_{name}"] = ssa.expand_kv_for_gqa(kv, h_q, shape[-2]).numpy()
        out[f"hq_{name}"] = np.array(h_q)
    np.savez_compressed(os.path.join(HERE, "gqa_expand.npz"), **out)


def main():
    import numpy as np
    import torch

    ssa = _import_reference()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    gqa_expand(ssa)
    if "--only" in sys.argv:
        return

    # ---------------- stage 1 + 2 ----------------
    torch.manual_seed(1234)
    n, h_q, h_kv, d, d_s, n_c, a, b, k = 96, 8, 2, 64, 16, 32, 8, 4, 16
    router = ssa.CodebookRouter(head_dim=d, route_dim=d_s, num_kv_heads=h_kv,
                                num_codebook=n_c, codes_per_key=b,
                                codes_per_query=a, top_k=k)
    q = torch.randn(n, h_q, d)
    kk = torch.randn(n, h_kv, d)
    mask = ssa.build_causal_mask(n)
    captured = {}
    orig = router._select_candidates

    def capture(q_full, k_full, q_code_scores, k_code_assign, top_q_codes, causal_mask):
        captured["q_code_scores"] = q_code_scores.detach().clone()
        captured["k_code_assign"] = k_code_assign.detach().clone()
        captured["top_q_codes"] = top_q_codes.detach().clone()
        return orig(q_full, k_full, q_code_scores, k_code_assign, top_q_codes, causal_mask)

    router._select_candidates = capture
    with torch.no_grad():
        idx = router(q, kk, causal_mask=mask, hard=True)
        cand = router._build_candidate_mask(captured["top_q_codes"], captured["k_code_assign"],
                                            n, h_kv, q.device)
    finite = (cand & mask[:, None, :]).sum(-1)                       # [n, h_kv]
    well_defined = finite >= min(k, n)
    np.savez_compressed(
        os.path.join(HERE, "stage1.npz"),
        q=q.numpy(), k=kk.numpy(),
        w_qr=router.W_qr.weight.detach().numpy(), w_kr=router.W_kr.weight.detach().numpy(),
        codebook=router.codebook.detach().numpy(),
        dims=np.array([n, h_q, h_kv, d, d_s, n_c, a, b, k]),
        q_code_scores=captured["q_code_scores"].numpy(),
        k_code_assign=captured["k_code_assign"].numpy(),
        top_q_codes=captured["top_q_codes"].numpy(),
        candidate_mask=np.packbits(cand.numpy().reshape(-1)),
        indices=idx.numpy(), well_defined=well_defined.numpy())

    # ---------------- stage 3, h_kv = 1 and 2 ----------------
    for name, hkv in (("stage3_h1", 1), ("stage3_h2", 2)):
        torch.manual_seed(99 + hkv)
        n3, hq3, d3, k3 = 40, 4, 16, 12
        q3 = torch.randn(n3, hq3, d3)
        k3t = torch.randn(n3, hkv, d3)
        v3 = torch.randn(n3, hkv, d3)
        idx3 = torch.randint(0, n3, (n3, hkv, k3))
        out = ssa.sparse_exact_attention(q3, k3t, v3, idx3)
        out_s = ssa.sparse_exact_attention(q3, k3t, v3, idx3, scale=2.5)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=q3.numpy(), k=k3t.numpy(),
                            v=v3.numpy(), indices=idx3.numpy(), out=out.numpy(),
                            out_scale=out_s.numpy())

    # ---------------- dense ----------------
    torch.manual_seed(7)
    q4, k4, v4 = torch.randn(48, 6, 16), torch.randn(48, 2, 16), torch.randn(48, 2, 16)
    out4 = ssa.dense_attention(q4, k4, v4, causal_mask=ssa.build_causal_mask(48))
    np.savez_compressed(os.path.join(HERE, "dense.npz"), q=q4.numpy(), k=k4.numpy(),
                        v=v4.numpy(), out=out4.numpy())

    # ---------------- module (SSAAttention with RoPE, h_kv = 1) ----------------
    torch.manual_seed(2024)
    hs, nq5, nkv5, d5, n5 = 128, 4, 1, 32, 64
    mod = ssa.SSAAttention(hidden_size=hs, num_q_heads=nq5, num_kv_heads=nkv5, head_dim=d5,
                           route_dim=8, num_codebook=16, codes_per_key=4,
                           codes_per_query=6, top_k=12)
    x = torch.randn(1, n5, hs)
    freqs = ssa.precompute_rope_freqs(d5, 2 * n5)
    seen = {}
    orig_fwd = mod.router.forward

    def capture_router(q_full, k_full, causal_mask=None, hard=True):
        seen["q"] = q_full.detach().clone()
        seen["k"] = k_full.detach().clone()
        out_idx = orig_fwd(q_full, k_full, causal_mask=causal_mask, hard=hard)
        seen["idx"] = out_idx.clone()
        return out_idx

    mod.router.forward = capture_router
    with torch.no_grad():
        y = mod(x, freqs=freqs)
    # well-defined rows: >= min(k, n) causal candidates
    r = mod.router
    with torch.no_grad():
        qr = r.W_qr(seen["q"]).view(n5, nkv5, nq5 // nkv5, -1).mean(2)
        kr = r.W_kr(seen["k"])
        cbn = torch.nn.functional.normalize(r.codebook, dim=-1)
        qs = torch.einsum("shd,hcd->shc", torch.nn.functional.normalize(qr, dim=-1), cbn)
        ks = torch.einsum("shd,hcd->shc", torch.nn.functional.normalize(kr, dim=-1), cbn)
        tq = qs.topk(r.codes_per_query, dim=-1).indices
        ka = ks.topk(r.codes_per_key, dim=-1).indices
        cm = r._build_candidate_mask(tq, ka, n5, nkv5, x.device)
    wd = ((cm & ssa.build_causal_mask(n5)[:, None, :]).sum(-1) >= min(r.top_k, n5)).all(-1)
    state = {kname: v.detach().numpy() for kname, v in mod.state_dict().items()}
    np.savez_compressed(os.path.join(HERE, "module.npz"), x=x.numpy(), y=y.numpy(),
                        freqs=freqs.numpy(), q_rope=seen["q"].numpy(), k_rope=seen["k"].numpy(),
                        indices=seen["idx"].numpy(), well_defined_rows=wd.numpy(),
                        dims=np.array([hs, nq5, nkv5, d5, n5, 8, 16, 4, 6, 12]),
                        **{"sd_" + kname.replace(".", "__"): v for kname, v in state.items()})
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
