"""Seeded synthetic inputs for the benchmark configurations.

The reference publishes no dataset for this path; these generators follow
the shapes and value distributions its benchmark configurations name:

* config 2 -- dense equivalence: Q/K/V ~ N(0, 1), k = n.
* config 3 -- op-level sweep: Q/K ~ N(0, 1) with 5% of keys replaced by one
  of 64 Gaussian centroids plus N(0, 0.1^2) noise (planted clusters, so that
  routing is non-trivial); V ~ N(0, 1).
* config 4 -- long single sequence: Q/K/V ~ N(0, 1).

Router weights: W_qr / W_kr xavier-uniform, codebook ~ N(0, 1/d_s).
"""

from __future__ import annotations

from dataclasses import dataclass, asdict

import torch


@dataclass
class Shape:
    n: int
    h_q: int
    h_kv: int
    d: int
    d_s: int
    n_codes: int
    a: int
    b: int
    top_k: int
    batch: int = 1
    causal: bool = True

    def asdict(self):
        return asdict(self)


CONFIG2 = Shape(n=4096, h_q=8, h_kv=2, d=64, d_s=32, n_codes=1024, a=16, b=4, top_k=4096)
CONFIG3 = Shape(n=32768, h_q=32, h_kv=8, d=128, d_s=32, n_codes=4096, a=16, b=4, top_k=256)
CONFIG4 = Shape(n=131072, h_q=32, h_kv=8, d=128, d_s=32, n_codes=8192, a=16, b=4, top_k=512)


def make_inputs(shape: Shape, seed: int = 0, dtype=torch.bfloat16, device="cuda", planted: bool = True,
                generate_on_device: bool = False):
    """Returns dict(q [B,n,h_q,d], k, v [B,n,h_kv,d], w_qr, w_kr [d_s,d] fp32,
    codebook [h_kv,N_c,d_s] fp32) from ``seed``, on ``device``.

    ``generate_on_device`` draws the numbers on ``device`` itself (fast for
    long sequences; the same seed gives the same values on every GPU) instead
    of on the host; the two give different numbers."""
    gen_dev = device if generate_on_device else "cpu"
    g = torch.Generator(device=gen_dev).manual_seed(seed)
    B, n = shape.batch, shape.n

    def randn(*s):
        return torch.randn(*s, generator=g, dtype=torch.float32, device=gen_dev)

    q = randn(B, n, shape.h_q, shape.d)
    k = randn(B, n, shape.h_kv, shape.d)
    v = randn(B, n, shape.h_kv, shape.d)
    if planted:
        n_planted = max(1, n // 20)
        cent = randn(64, shape.d)
        for bi in range(B):
            for h in range(shape.h_kv):
                rows = torch.randperm(n, generator=g, device=gen_dev)[:n_planted]
                which = torch.randint(0, 64, (n_planted,), generator=g, device=gen_dev)
                k[bi, rows, h] = cent[which] + 0.1 * randn(n_planted, shape.d)
    bound = (6.0 / (shape.d + shape.d_s)) ** 0.5
    w_qr = (torch.rand(shape.d_s, shape.d, generator=g, device=gen_dev) * 2 - 1) * bound
    w_kr = (torch.rand(shape.d_s, shape.d, generator=g, device=gen_dev) * 2 - 1) * bound
    cb = randn(shape.h_kv, shape.n_codes, shape.d_s) / shape.d_s ** 0.5
    out = dict(q=q.to(dtype), k=k.to(dtype), v=v.to(dtype), w_qr=w_qr, w_kr=w_kr, codebook=cb)
    return {kk: t.to(device) for kk, t in out.items()}
