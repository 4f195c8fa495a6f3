"""Token-by-token SSA decoding over a growing key/value cache.

Each step appends the new position's key and value, assigns the key its
codes once (``ssa_code_assign`` on that row only), adds the key's ``b``
entries to the cache's code->key index (``ssa_decode_index_append``: one
small launch, whatever the number of cached keys), routes the new query
against the index (``ssa_decode_route``, ``q_offset`` = the query's
position) and attends over the selected keys (``ssa_sparse_attn``).

The index keeps free slots after every bucket (``ssa_decode_index_build``
gives each bucket ``max(slack, its size)`` of them), so appends never move
entries.  The device tracks the fewest free slots of any bucket; its value
is read back without stalling the host, and since a key's codes are
distinct, appending ``t`` keys takes at most ``t`` slots of any bucket: the
cache rebuilds the index (an O(n) pass, with more room) only when the last
value it saw leaves less room than the keys it is about to append.  Buckets
grow their room with their size, so rebuilds become rare as the cache grows.

The reference has no decode path (its design notes ask for an index
maintained incrementally, ``ssa_design.md``); a step computes what
``CodebookRouter.forward`` + ``sparse_exact_attention`` compute for the last
row of the sequence so far (``ssa/router.py:73-149``,
``ssa/attention.py:12-115``).  While fewer than ``top_k`` keys are cached the
indices are zero-padded as the reference pads ``k > n``
(``ssa/router.py:206-211``), so from position ``top_k - 1`` on a step equals
the full-sequence forward's row.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib as L
from . import _status as S
from . import ops

# keys appended at once above which a rebuild is cheaper than appending
_BULK = 64


class DecodeCache:
    """Keys, values, key codes and the code->key index of ``batch``
    sequences, up to ``capacity`` positions each, on one GPU."""

    def __init__(self, router, batch: int, capacity: int, num_q_heads: int, dtype=torch.bfloat16,
                 device="cuda", slack: int = 32):
        self.router = router
        self.batch, self.capacity = batch, capacity
        self.h_q, self.h_kv, self.d = num_q_heads, router.num_kv_heads, router.head_dim
        if self.h_q % self.h_kv:
            raise ValueError("num_q_heads must be divisible by num_kv_heads")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        shape = (batch, capacity, self.h_kv, self.d)
        self.k = torch.empty(shape, dtype=dtype, device=dev)
        self.v = torch.empty(shape, dtype=dtype, device=dev)
        b, n_codes = router.codes_per_key, router.num_codebook
        self.codes = torch.zeros((batch, capacity, self.h_kv, b), dtype=torch.int32, device=dev)
        self.n = 0
        # the index: free slots after every bucket
        self.slack = slack
        cap = int(L.lib().ssa_decode_index_capacity(capacity, b, n_codes, slack))
        self.ix_start = torch.zeros((batch, self.h_kv, n_codes + 1), dtype=torch.int32, device=dev)
        self.ix_end = torch.zeros((batch, self.h_kv, n_codes + 1), dtype=torch.int32, device=dev)
        self.ix_keys = torch.empty((batch, self.h_kv, cap), dtype=torch.int32, device=dev)
        self.ix_codes = (torch.empty((batch, self.h_kv, cap, 4), dtype=torch.int32, device=dev)
                         if b == 4 else None)
        self.min_free = torch.zeros(1, dtype=torch.int32, device=dev)
        ix = L.SsaDecodeIndex()
        ix.bucket_start, ix.bucket_end = self.ix_start.data_ptr(), self.ix_end.data_ptr()
        ix.bucket_keys = self.ix_keys.data_ptr()
        ix.bucket_codes = self.ix_codes.data_ptr() if self.ix_codes is not None else None
        ix.entry_capacity, ix.slack, ix.min_free = cap, slack, self.min_free.data_ptr()
        ix.k_codes_stride_b = capacity * self.h_kv * b
        self.index = ix
        self._built = False
        self._free_lb = 0              # a lower bound on the free slots of every bucket
        self._mf_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._mf_read = None           # (event, keys indexed when the copy was queued)
        self.rebuilds = 0
        self._ws = None

    # -- argument blocks -------------------------------------------------
    def _args(self, n: int, q: Optional[torch.Tensor] = None, indices: Optional[torch.Tensor] = None,
              q_offset: int = 0) -> L.SsaRouteArgs:
        r = self.router
        k = self.k[:, :n]
        w_qr, w_kr, cb = ops._prep_weights(r.W_qr.weight.detach(), r.W_kr.weight.detach(), r.codebook.detach(),
                                           k.dtype)
        self._keep = (w_qr, w_kr, cb)
        qq = q if q is not None else k
        args = ops.route_args(qq, k, w_qr, w_kr, cb, r.codes_per_query, r.codes_per_key, r.top_k, True,
                              float(r.temperature), q_offset, indices, False, None, None, None)
        if q is None:
            args.n_q = 1
        args.k_codes = self.codes.data_ptr()
        return args

    def _workspace(self) -> torch.Tensor:
        if self._ws is None:
            # sized for a full cache and one query row: covers every call below
            self._ws = ops.workspace(self._args(self.capacity), self.device)
        return self._ws

    # -- the index -------------------------------------------------------
    def _refresh_bound(self) -> None:
        """The fewest free slots, from the last read-back: ``n_at`` keys were
        indexed when it was queued, ``self.n`` are now, so at most
        ``self.n - n_at`` slots of any bucket were taken since.  When the host
        runs ahead of the GPU the read-back may still be in flight; waiting
        for it (a few steps of GPU work) is cheaper than an O(n) rebuild."""
        if self._mf_read is None:
            return
        ev, n_at = self._mf_read
        ev.synchronize()
        self._free_lb = int(self._mf_host[0]) - (self.n - n_at)
        self._mf_read = None

    def _index(self, first: int, t: int) -> None:
        lib, st = L.lib(), torch.cuda.current_stream(self.device).cuda_stream
        n = first + t
        if self._built and self._free_lb < t:
            self._refresh_bound()
        slot = S.acquire(self.device)
        args = self._args(n)
        args.status = slot.ptr if slot is not None else None
        if not self._built or self._free_lb < t or t > _BULK:
            ws = self._workspace()
            L.check("ssa_decode_index_build",
                    lib.ssa_decode_index_build(ctypes.byref(args), ctypes.byref(self.index), ws.data_ptr(),
                                               ws.numel(), st))
            self._built, self._free_lb = True, self.slack
            self.rebuilds += 1
        else:
            L.check("ssa_decode_index_append",
                    lib.ssa_decode_index_append(ctypes.byref(args), ctypes.byref(self.index), first, t, st))
            self._free_lb -= t
        S.release(slot, "ssa_decode_index", S.route_error)
        # the fewest free slots after this update, read back without waiting
        self._mf_host.copy_(self.min_free, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._mf_read = (ev, n)

    # -- public ------------------------------------------------------------
    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> None:
        """Adds ``t`` positions: ``k_new``, ``v_new`` ``[batch, t, h_kv, d]``."""
        t = k_new.shape[1]
        if self.n + t > self.capacity:
            raise ValueError(f"cache full: {self.n} + {t} > {self.capacity}")
        s = slice(self.n, self.n + t)
        self.k[:, s] = k_new
        self.v[:, s] = v_new
        self.codes[:, s] = self.router.key_codes(self.k[:, s])
        first = self.n
        self.n += t
        with torch.cuda.device(self.device):
            self._index(first, t)

    def step(self, q_new: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             scale: Optional[float] = None) -> torch.Tensor:
        """One decoding step: appends position ``n`` (``k_new``, ``v_new``
        ``[batch, 1, h_kv, d]``) and returns the attention output of its query
        ``q_new [batch, 1, h_q, d]`` over the routed keys, ``[batch, 1, h_q, d]``."""
        self.append(k_new, v_new)
        n = self.n
        q = ops._last_contig(q_new.to(self.k.dtype))
        idx = torch.empty((self.batch, 1, self.h_kv, self.router.top_k), dtype=torch.int32, device=self.device)
        args = self._args(n, q=q, indices=idx, q_offset=n - 1)
        slot = S.acquire(self.device)
        args.status = slot.ptr if slot is not None else None
        ws = self._workspace()
        with torch.cuda.device(self.device):
            L.check("ssa_decode_route",
                    L.lib().ssa_decode_route(ctypes.byref(args), ctypes.byref(self.index), ws.data_ptr(), ws.numel(),
                                             torch.cuda.current_stream(self.device).cuda_stream))
            S.release(slot, "ssa_decode_route", S.route_error)
        if scale is None:
            scale = math.sqrt(self.d)
        return ops.sparse_attn(q, self.k[:, :n], self.v[:, :n], idx, float(scale), True, n - 1)
