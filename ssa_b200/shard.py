"""One long sequence over several GPUs: the query-sharded SSA forward.

One process per GPU (``torch.distributed``, NCCL over NVLink).  The ``n``
positions of the sequence are cut into ``2 * W`` equal blocks and rank ``r``
owns blocks ``r`` and ``2W - 1 - r`` (a zig-zag assignment).  Under the causal
mask a query at position ``i`` has candidates among ``i + 1`` keys only, so
the routing work grows with the position; pairing an early block with a late
one gives every rank the same share.  A rank holds the query, key and value
rows of its two blocks, in that order.

Per forward (:func:`sharded_forward`):

1. key codes of the rank's own key rows -- the code assignment of a key
   depends on that key alone (``ssa/router.py:114-130``);
2. the one exchange step: all-gather of the key codes, K and V into
   full-sequence buffers, in that order (collectives run in issue order, so
   the small code gather is issued first);
3. the code->key index of all ``n`` keys, built once as soon as the codes
   have arrived -- K and V are still moving meanwhile;
4. for each of its two blocks, routing of the block's queries against all
   ``n`` keys with the gathered codes and the index (``q_offset`` = the
   block's start) -- V is still arriving meanwhile -- then sparse attention
   over the selected keys.

The reference has no distributed code; this follows the per-query
independence of ``CodebookRouter.forward`` (``ssa/router.py:73-149``) and
``sparse_exact_attention`` (``ssa/attention.py:12-115``).
"""

from __future__ import annotations

import math
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


def zigzag_blocks(n: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """``[(start, length), (start, length)]`` of the two blocks rank ``rank``
    owns; ``n`` must be a multiple of ``2 * world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n % (2 * world):
        raise ValueError(f"sequence length {n} must be a multiple of 2 * world_size = {2 * world}")
    blk = n // (2 * world)
    return [(rank * blk, blk), ((2 * world - 1 - rank) * blk, blk)]


def local_rows(x: torch.Tensor, world: int, rank: int, dim: int = 1) -> torch.Tensor:
    """The rows of a full-sequence tensor that rank ``rank`` holds: its two
    blocks along ``dim``, concatenated."""
    blocks = zigzag_blocks(x.shape[dim], world, rank)
    return torch.cat([x.narrow(dim, s, ln) for s, ln in blocks], dim=dim)


def _block_order(world: int) -> torch.Tensor:
    """Gathered slot (rank * 2 + which) of every sequence block 0 .. 2W-1."""
    order = torch.empty(2 * world, dtype=torch.long)
    for r in range(world):
        order[r] = 2 * r
        order[2 * world - 1 - r] = 2 * r + 1
    return order


def gather_sequence(local: torch.Tensor, world: int, group=None, async_op: bool = False):
    """All-gather the zig-zag shards ``local [B, 2*blk, ...]`` of every rank
    into the full sequence ``[B, 2*W*blk, ...]`` (sequence on dim 1).

    With ``async_op`` returns ``(work, finish)``: wait on ``work``, then call
    ``finish()`` for the full tensor."""
    B, rows = local.shape[0], local.shape[1]
    if rows % 2:
        raise ValueError("a rank holds two blocks of equal length")
    blk = rows // 2
    tail = tuple(local.shape[2:])
    # [2, B, blk, ...]: the rank's two blocks, each contiguous
    mine = local.reshape(B, 2, blk, *tail).transpose(0, 1).contiguous()
    buf = torch.empty((world * 2, B, blk) + tail, dtype=local.dtype, device=local.device)
    work = dist.all_gather_into_tensor(buf, mine, group=group, async_op=async_op)

    def finish() -> torch.Tensor:
        order = _block_order(world).to(local.device)
        full = buf.index_select(0, order)                                 # [2W, B, blk, ...]
        return full.transpose(0, 1).reshape((B, 2 * world * blk) + tail)

    if async_op:
        return work, finish
    return finish()


def sharded_forward(router, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                    group=None, causal: bool = True, scale: Optional[float] = None,
                    code_fn: Optional[Callable] = None, index_fn: Optional[Callable] = None,
                    route_fn: Optional[Callable] = None, attn_fn: Optional[Callable] = None) -> torch.Tensor:
    """SSA forward of this rank's query rows of one sequence.

    ``q_local [B, 2*blk, h_q, d]``, ``k_local``/``v_local [B, 2*blk, h_kv, d]``
    are the rows of this rank's two zig-zag blocks (:func:`local_rows`);
    returns the attention output for those rows, ``[B, 2*blk, h_q, d]``.

    ``code_fn(k) -> codes``, ``index_fn(codes) -> index``,
    ``route_fn(q_block, k, codes, index, q_offset) -> indices`` and
    ``attn_fn(q_block, k, v, indices, q_offset) -> out`` default to the
    sm_100a kernels (:meth:`CodebookRouter.key_codes`,
    :meth:`CodebookRouter.key_index`, :meth:`CodebookRouter.route_with_index`,
    sparse attention); they are parameters so that the exchange logic can be
    checked on CPU ranks."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    rows = q_local.shape[1]
    n = rows * world
    blocks = zigzag_blocks(n, world, rank)
    if scale is None:
        scale = math.sqrt(q_local.shape[-1])
    if code_fn is None:
        code_fn = router.key_codes
    if index_fn is None:
        index_fn = router.key_index
    if route_fn is None:
        def route_fn(qb, k, codes, index, q_offset):
            return router.route_with_index(qb, k, codes, index, causal=causal, q_offset=q_offset,
                                           index_dtype=torch.int32)
    if attn_fn is None:
        from . import ops

        def attn_fn(qb, k, v, idx, q_offset):
            return ops.sparse_attn(qb, k, v, idx, float(scale), bool(causal), int(q_offset))

    # the exchange.  The codes go first: the index built from them needs
    # neither K nor V, so it is built while K and V are still moving (a code
    # gather issued after them would wait for both).
    codes_local = code_fn(k_local)
    c_work, c_finish = gather_sequence(codes_local, world, group, async_op=True)
    k_work, k_finish = gather_sequence(k_local, world, group, async_op=True)
    v_work, v_finish = gather_sequence(v_local, world, group, async_op=True)
    c_work.wait()
    codes = c_finish()
    index = index_fn(codes)
    k_work.wait()
    k_full = k_finish()
    qbs = [q_local[:, which * length:(which + 1) * length] for which, (start, length) in enumerate(blocks)]
    idxs = [route_fn(qb, k_full, codes, index, start) for qb, (start, _) in zip(qbs, blocks)]
    v_work.wait()
    v_full = v_finish()
    outs = [attn_fn(qb, k_full, v_full, idx, start) for qb, idx, (start, _) in zip(qbs, idxs, blocks)]
    return torch.cat(outs, dim=1)
