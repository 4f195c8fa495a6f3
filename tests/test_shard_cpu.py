"""Query-sharded forward of one sequence (ssa_b200.shard) on CPU ranks.

World sizes 2 and 3 run as spawned ``gloo`` processes.  The per-block compute
is injected with the CPU oracle, so these tests check the exchange logic --
the zig-zag block assignment, the all-gather of K, V and key codes back into
sequence order, and the ``q_offset`` of each block -- against a
single-process oracle run of the whole sequence.  The GPU kernels behind the
default compute functions are covered by the ``gpu`` tests.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ssa_oracle as O
from ssa_b200 import shard

N, HQ, HKV, D, DS, NC, A, B, TOPK = 96, 4, 2, 16, 8, 24, 3, 2, 20


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(seed=0):
    rng = np.random.default_rng(seed)
    q = rng.integers(-3, 4, size=(N, HQ, D)).astype(np.float64)
    k = rng.integers(-3, 4, size=(N, HKV, D)).astype(np.float64)
    v = rng.standard_normal((N, HKV, D))
    w_qr = rng.standard_normal((DS, D))
    w_kr = rng.standard_normal((DS, D))
    cb = rng.standard_normal((HKV, NC, DS))
    return q, k, v, w_qr, w_kr, cb


def _oracle_full(p):
    q, k, v, w_qr, w_kr, cb = p
    qc, kc = O.route_codes(q, k, w_qr, w_kr, cb, A, B)
    idx = O.select_topk_dense(q, k, qc, kc, TOPK, causal=True)
    return O.sparse_attention(q, k, v, idx, causal=True)


def _oracle_fns(p):
    _, _, _, w_qr, w_kr, cb = p

    def code_fn(k_local):                                  # [1, rows, h_kv, d] -> [1, rows, h_kv, b]
        kl = k_local[0].numpy()
        _, k_route = O.route_vectors(np.zeros((kl.shape[0], HQ, D)), kl, w_qr, w_kr)
        return torch.from_numpy(O.stable_topk(O.code_scores(k_route, cb), B).astype(np.int32))[None]

    def query_code_fn(ql):                                 # [1, rows, h_q, d] -> [1, rows, h_kv, a]
        qn = ql[0].numpy()
        q_route, _ = O.route_vectors(qn, np.zeros((qn.shape[0], HKV, D)), w_qr, w_kr)
        return torch.from_numpy(O.stable_topk(O.code_scores(q_route, cb), A).astype(np.int32))[None]

    def route_fn(ql, k, qc, codes, index, blocks):
        outs, r0 = [], 0
        for q_offset, ln in blocks:                           # the rank's blocks, in position order
            qn = ql[0, r0:r0 + ln].numpy()
            outs.append(O.select_topk_dense(qn, k[0].numpy(), qc[0, r0:r0 + ln].numpy(), codes[0].numpy(),
                                            TOPK, causal=True, q_start=q_offset))
            r0 += ln
        return torch.from_numpy(np.concatenate(outs))[None]

    def attn_fn(ql, k, v, idx, blocks):
        pos = np.concatenate([np.arange(s, s + ln) for s, ln in blocks])
        out = O.sparse_attention(ql[0].numpy(), k[0].numpy(), v[0].numpy(), idx[0].numpy(),
                                 causal=True, positions=pos)
        return torch.from_numpy(out)[None]

    return code_fn, query_code_fn, route_fn, attn_fn


def _worker(rank, world, port, task, result_dir, folds=1):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if task == "gather":
            full = torch.arange(2 * N * HKV * 3, dtype=torch.int32).reshape(2, N, HKV, 3)
            local = shard.local_rows(full, world, rank, folds=folds)
            got = shard.gather_sequence(local, world, folds=folds)
            ok = torch.equal(got, full)
        else:
            p = _problem()
            q, k, v = (torch.from_numpy(x)[None] for x in p[:3])
            ql, kl, vl = (shard.local_rows(x, world, rank, folds=folds) for x in (q, k, v))
            code_fn, query_code_fn, route_fn, attn_fn = _oracle_fns(p)
            out = shard.sharded_forward(None, ql, kl, vl, folds=folds, code_fn=code_fn,
                                        query_code_fn=query_code_fn, index_fn=lambda c: None,
                                        route_fn=route_fn, attn_fn=attn_fn,
                                        kv_after_query_codes=task == "forward_late_kv",
                                        v_after_query_codes=task == "forward_late_v")
            want = shard.local_rows(torch.from_numpy(_oracle_full(p))[None], world, rank, folds=folds)
            ok = out.shape == want.shape and torch.allclose(out, want, rtol=0, atol=1e-12)
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def _run(world, task, tmp_path, folds=1):
    mp.spawn(_worker, args=(world, _free_port(), task, str(tmp_path), folds), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", f"rank {r} of {world}"


def test_zigzag_blocks_cover_the_sequence_and_balance_causal_work():
    n = 96
    for world in (1, 2, 3, 4):
        seen = np.zeros(n, dtype=int)
        work = []
        for r in range(world):
            blocks = shard.zigzag_blocks(n, world, r)
            assert len(blocks) == 2 and blocks[0][1] == blocks[1][1] == n // (2 * world)
            w = 0
            for s, ln in blocks:
                seen[s:s + ln] += 1
                w += sum(i + 1 for i in range(s, s + ln))       # causal keys per query
            work.append(w)
        assert (seen == 1).all()
        assert len(set(work)) == 1                            # every rank the same causal work
    with pytest.raises(ValueError):
        shard.zigzag_blocks(100, 3, 0)


def test_folded_zigzag_blocks_ascend_and_cover_the_sequence():
    n = 96
    for world, folds in ((1, 2), (2, 2), (3, 2), (2, 3)):
        seen = np.zeros(n, dtype=int)
        for r in range(world):
            blocks = shard.zigzag_blocks(n, world, r, folds)
            assert len(blocks) == 2 * folds
            assert [s for s, _ in blocks] == sorted(s for s, _ in blocks)
            for s, ln in blocks:
                seen[s:s + ln] += 1
        assert (seen == 1).all()


@pytest.mark.parametrize("world,folds", [(2, 1), (3, 1), (2, 2)])
def test_gather_sequence_round_trip(world, folds, tmp_path):
    _run(world, "gather", tmp_path, folds)


@pytest.mark.parametrize("world,folds", [(2, 1), (3, 1), (2, 2)])
def test_sharded_forward_matches_single_process(world, folds, tmp_path):
    _run(world, "forward", tmp_path, folds)


@pytest.mark.parametrize("task", ["forward_late_kv", "forward_late_v"])
def test_sharded_forward_with_late_gathers(task, tmp_path):
    """K and V (or V alone) gathered after the query codes: the same output."""
    _run(2, task, tmp_path, 2)
