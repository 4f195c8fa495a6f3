"""Query-sharded forward of one sequence on 2 GPUs (NCCL), against one GPU.

Each rank holds the rows of its two zig-zag blocks, assigns codes to its own
keys, all-gathers K, V and the key codes, and routes and attends its own
queries.  Every per-row computation is the same as in the single-GPU run, so
the outputs must agree exactly.  Skipped with fewer than 2 GPUs.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    from datetime import timedelta

    import ssa_b200 as ssa
    from ssa_b200 import ops, shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        torch.manual_seed(0)
        router = ssa.CodebookRouter(head_dim=128, route_dim=32, num_kv_heads=4, num_codebook=1024,
                                    codes_per_key=4, codes_per_query=8, top_k=128).to(dev)
        g = torch.Generator(device="cpu").manual_seed(1)
        n = 4096
        q = torch.randn((1, n, 16, 128), generator=g).to(dev, torch.bfloat16)
        k = torch.randn((1, n, 4, 128), generator=g).to(dev, torch.bfloat16)
        v = torch.randn((1, n, 4, 128), generator=g).to(dev, torch.bfloat16)
        # single-GPU result of the whole sequence, on this rank's GPU
        idx, _, _, _ = router.route(q, k, causal=True, index_dtype=torch.int32)
        full = ops.sparse_attn(q, k, v, idx, 128 ** 0.5, True, 0)
        ok = True
        for folds in (1, 2, 2):            # the repeat reuses the side stream and the cached block order
            ql, kl, vl = (shard.local_rows(x, world, rank, folds=folds) for x in (q, k, v))
            out = shard.sharded_forward(router, ql, kl, vl, causal=True, folds=folds)
            torch.cuda.synchronize(dev)
            ok = ok and torch.equal(out, shard.local_rows(full, world, rank, folds=folds))
        ssa.check_errors(dev)
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_sharded_forward_two_gpus_matches_one_gpu(tmp_path):
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert (tmp_path / f"rank{r}").read_text() == "ok", f"rank {r}"
