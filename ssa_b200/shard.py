"""One long sequence over several GPUs: the query-sharded SSA forward.

One process per GPU (``torch.distributed``, NCCL over NVLink).  The ``n``
positions of the sequence are cut into ``2 * folds * W`` equal blocks and, in
each of the ``folds`` passes over ``2 W`` consecutive blocks, rank ``r`` owns
blocks ``r`` and ``2W - 1 - r`` (a zig-zag assignment).  Under the causal
mask a query at position ``i`` has candidates among ``i + 1`` keys only, so
the routing work grows with the position; pairing an early block with a late
one gives every rank about the same share, and more folds (smaller blocks)
even out the part of the cost that does not grow linearly.  A rank holds the
query, key and value rows of its blocks, in position order.

Per forward (:func:`sharded_forward`):

1. key codes of the rank's own key rows -- the code assignment of a key
   depends on that key alone (``ssa/router.py:114-130``);
2. the one exchange step: all-gather of the key codes, K and V into
   full-sequence buffers, in that order (collectives run in issue order, so
   the small code gather is issued first);
3. the query codes of the rank's own query rows, which need nothing from
   the other ranks (``ssa/router.py:102-112,130``), while the gathers move;
4. the code->key index of all ``n`` keys, built once as soon as the codes
   have arrived;
5. one candidate-selection call for all of the rank's query blocks against
   all ``n`` keys (query segments: each block at its own sequence position)
   -- V is still arriving meanwhile -- then one sparse-attention call over
   the selected keys.

On GPUs the gathered rows are put back in sequence order on a side stream,
so that the copies overlap the routing kernels.

The reference has no distributed code; this follows the per-query
independence of ``CodebookRouter.forward`` (``ssa/router.py:73-149``) and
``sparse_exact_attention`` (``ssa/attention.py:12-115``).
"""

from __future__ import annotations

import math
from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist


def zigzag_blocks(n: int, world: int, rank: int, folds: int = 1) -> List[Tuple[int, int]]:
    """``[(start, length), ...]`` of the ``2 * folds`` blocks rank ``rank``
    owns, in ascending positions; ``n`` must be a multiple of ``2 * folds * world``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if folds < 1:
        raise ValueError(f"folds must be >= 1, got {folds}")
    if n % (2 * folds * world):
        raise ValueError(f"sequence length {n} must be a multiple of 2 * folds * world_size = {2 * folds * world}")
    blk = n // (2 * folds * world)
    out = []
    for f in range(folds):
        base = f * 2 * world
        out += [((base + rank) * blk, blk), ((base + 2 * world - 1 - rank) * blk, blk)]
    return out


def local_rows(x: torch.Tensor, world: int, rank: int, dim: int = 1, folds: int = 1) -> torch.Tensor:
    """The rows of a full-sequence tensor that rank ``rank`` holds: its blocks
    along ``dim``, concatenated in position order."""
    blocks = zigzag_blocks(x.shape[dim], world, rank, folds)
    return torch.cat([x.narrow(dim, s, ln) for s, ln in blocks], dim=dim)


def _block_order(world: int, folds: int = 1) -> torch.Tensor:
    """Gathered slot (rank * 2 * folds + which) of every sequence block."""
    per = 2 * folds
    order = torch.empty(per * world, dtype=torch.long)
    for r in range(world):
        for f in range(folds):
            base = f * 2 * world
            order[base + r] = r * per + 2 * f
            order[base + 2 * world - 1 - r] = r * per + 2 * f + 1
    return order


_orders = {}


def _device_block_order(world: int, folds: int, device: torch.device) -> torch.Tensor:
    """:func:`_block_order` kept on the device, so that a forward issues no
    host-to-device copy."""
    key = (world, folds, str(device))
    if key not in _orders:
        _orders[key] = _block_order(world, folds).to(device)
    return _orders[key]


def gather_sequence(local: torch.Tensor, world: int, group=None, async_op: bool = False, folds: int = 1):
    """All-gather the zig-zag shards ``local [B, 2*folds*blk, ...]`` of every
    rank into the full sequence ``[B, 2*folds*W*blk, ...]`` (sequence on dim 1).

    With ``async_op`` returns ``(work, finish)``: wait on ``work``, then call
    ``finish()`` for the full tensor (on any stream: the gathered buffer is
    marked as used by the stream ``finish`` runs on)."""
    B, rows = local.shape[0], local.shape[1]
    per = 2 * folds
    if rows % per:
        raise ValueError(f"a rank holds {per} blocks of equal length")
    blk = rows // per
    tail = tuple(local.shape[2:])
    # [per, B, blk, ...]: the rank's blocks, each contiguous
    mine = local.reshape(B, per, blk, *tail).transpose(0, 1).contiguous()
    buf = torch.empty((world * per, B, blk) + tail, dtype=local.dtype, device=local.device)
    work = dist.all_gather_into_tensor(buf, mine, group=group, async_op=async_op)

    def finish() -> torch.Tensor:
        if buf.is_cuda:
            buf.record_stream(torch.cuda.current_stream(buf.device))
            order = _device_block_order(world, folds, buf.device)
        else:
            order = _block_order(world, folds)
        full = buf.index_select(0, order)                                 # [per*W, B, blk, ...]
        return full.transpose(0, 1).reshape((B, per * world * blk) + tail)

    if async_op:
        return work, finish
    return finish()


_side_streams = {}


def _arrive(work, finish, side):
    """Wait for one all-gather and put its rows in sequence order.  On a GPU
    both happen on the side stream ``side`` and the caller's stream waits for
    them only where it uses the result (:func:`_use`); on CPU ranks, here."""
    if side is None:
        work.wait()
        return finish(), None
    main = torch.cuda.current_stream(side.device)
    with torch.cuda.stream(side):
        work.wait()
        full = finish()
        ready = torch.cuda.Event()
        ready.record(side)
    full.record_stream(main)
    return full, ready


def _use(x, ready):
    """``x`` from :func:`_arrive`, once the current stream may read it."""
    if ready is not None:
        torch.cuda.current_stream(x.device).wait_event(ready)
    return x


def sharded_forward(router, q_local: torch.Tensor, k_local: torch.Tensor, v_local: torch.Tensor,
                    group=None, causal: bool = True, scale: Optional[float] = None, folds: int = 1,
                    code_fn: Optional[Callable] = None, query_code_fn: Optional[Callable] = None,
                    index_fn: Optional[Callable] = None, route_fn: Optional[Callable] = None,
                    attn_fn: Optional[Callable] = None, kv_after_query_codes: bool = False,
                    v_after_query_codes: bool = False, marks: Optional[list] = None) -> torch.Tensor:
    """SSA forward of this rank's query rows of one sequence.

    ``q_local [B, rows, h_q, d]``, ``k_local``/``v_local [B, rows, h_kv, d]``
    are the rows of this rank's ``2 * folds`` zig-zag blocks
    (:func:`local_rows`); returns the attention output for those rows,
    ``[B, rows, h_q, d]``.

    ``code_fn(k) -> key codes``, ``query_code_fn(q_local) -> query codes``,
    ``index_fn(codes) -> index``,
    ``route_fn(q_local, k, q_codes, codes, index, blocks) -> indices`` and
    ``attn_fn(q_local, k, v, indices, blocks) -> out`` (``blocks`` =
    ``[(start, length), ...]`` of the local rows, ascending) default to the
    sm_100a kernels (:meth:`CodebookRouter.key_codes`, ``ssa_query_codes``,
    :meth:`CodebookRouter.key_index`, candidate selection and sparse attention
    over query segments); they are parameters so that the exchange logic can
    be checked on CPU ranks."""
    from . import ops

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    rows = q_local.shape[1]
    n = rows * world
    blocks = zigzag_blocks(n, world, rank, folds)
    if scale is None:
        scale = math.sqrt(q_local.shape[-1])
    if code_fn is None:
        code_fn = router.key_codes
    if query_code_fn is None:
        def query_code_fn(ql):
            return ops.query_codes(ql, router.W_qr.weight, router.codebook, router.codes_per_query,
                                   router.num_kv_heads, float(router.temperature))
    if index_fn is None:
        index_fn = router.key_index
    if route_fn is None:
        def route_fn(ql, k, qc, codes, index, blks):
            return ops.select_candidates_segments(ql, k, qc, codes, index[0], index[1], router.top_k,
                                                  bool(causal), blks)
    if attn_fn is None:
        def attn_fn(ql, k, v, idx, blks):
            return ops.sparse_attn_segments(ql, k, v, idx, float(scale), bool(causal), blks)

    side = None
    if q_local.is_cuda:
        dev = q_local.device
        if dev not in _side_streams:
            _side_streams[dev] = torch.cuda.Stream(dev, priority=-1)
        side = _side_streams[dev]
        side.wait_stream(torch.cuda.current_stream(dev))

    # the exchange.  The codes go first: the index built from them needs
    # neither K nor V.  The query codes need nothing from the other ranks and
    # are computed while all three gathers are in flight; the reordering of
    # the gathered rows runs on a side stream, overlapped with routing.
    # With kv_after_query_codes the K and V gathers are issued after the query
    # codes (with v_after_query_codes only the V gather): the codebook-scoring
    # kernel keeps one CTA on every SM for its whole run, and collective
    # kernels launched before it hold SMs it then waits for; V is read only by
    # the attention, so its gather can move during the candidate selection.
    # `marks` (GPU ranks only): a list that receives (phase, CUDA event) pairs
    # recorded on the current stream at the end of each phase.
    def mark(name):
        if marks is not None and side is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(q_local.device))
            marks.append((name, ev))

    mark("start")
    codes_local = code_fn(k_local)
    mark("key codes")
    if kv_after_query_codes or v_after_query_codes:
        early = (codes_local,) if kv_after_query_codes else (codes_local, k_local)
        gathers = [gather_sequence(x, world, group, async_op=True, folds=folds) for x in early]
        q_codes = query_code_fn(q_local)
        late = (k_local, v_local) if kv_after_query_codes else (v_local,)
        gathers += [gather_sequence(x, world, group, async_op=True, folds=folds) for x in late]
    else:
        gathers = [gather_sequence(x, world, group, async_op=True, folds=folds)
                   for x in (codes_local, k_local, v_local)]
        q_codes = query_code_fn(q_local)
    mark("query codes")
    (codes, c_ready), (k_full, k_ready), (v_full, v_ready) = (_arrive(w, f, side) for w, f in gathers)
    index = index_fn(_use(codes, c_ready))
    mark("codes arrive + index")
    k_full = _use(k_full, k_ready)
    mark("K arrives")
    idx = route_fn(q_local, k_full, q_codes, codes, index, blocks)
    mark("candidates")
    v_full = _use(v_full, v_ready)
    mark("V arrives")
    out = attn_fn(q_local, k_full, v_full, idx, blocks)
    mark("attention")
    return out
