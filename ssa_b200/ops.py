"""PyTorch custom ops over the C ABI of libssa_sm100a.so.

Each op takes CUDA tensors, allocates its outputs (and, for the router, its
workspace) from the PyTorch caching allocator, and calls the library on the
current CUDA stream.  CPU tensors raise: there is no CPU path.

Ops (namespace ``ssa_b200``):
    route(q, k, w_qr, w_kr, codebook, a, b, top_k, causal, temperature,
          q_offset, index_i64) -> (indices, q_codes, k_codes, cand_counts)
    code_assign(k, w_kr, codebook, b, temperature) -> k_codes
    sparse_attn(q, k, v, indices, scale, causal, q_offset) -> out

``q`` is ``[B, n_q, h_q, d]``, ``k``/``v`` are ``[B, n, h_kv, d]``, indices
``[B, n_q, h_kv, top_k]``; the public API in :mod:`ssa_b200` adds the
reference's unbatched ``[n, h, d]`` forms.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib as L
from . import _status as S

_DT = {torch.float32: L.SSA_F32, torch.bfloat16: L.SSA_BF16, torch.float16: L.SSA_F16}


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if t.device.type != "cuda":
            raise RuntimeError("ssa_b200 ops need CUDA tensors (sm_100a); got a tensor on "
                               f"{t.device}. There is no CPU implementation.")
        if t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; use float32, bfloat16 or float16") from None


def _last_contig(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def route_args(q, k, w_qr, w_kr, codebook, a, b, top_k, causal, temperature, q_offset,
               indices=None, index_i64=True, q_codes=None, k_codes=None, cand_counts=None):
    """Fill an :class:`SsaRouteArgs` from 4-D tensors (no launch)."""
    B, n_q, h_q, d = q.shape
    _, n, h_kv, _ = k.shape
    cb = codebook if codebook.dim() == 3 else codebook.unsqueeze(0)
    args = L.SsaRouteArgs()
    args.batch, args.n, args.n_q, args.q_offset = B, n, n_q, q_offset
    args.h_q, args.h_kv, args.d, args.d_s = h_q, h_kv, d, w_kr.shape[0]
    args.n_codes, args.a, args.b, args.top_k = cb.shape[1], a, b, top_k
    args.causal, args.temperature = int(bool(causal)), float(temperature)
    args.dtype, args.w_dtype, args.codebook_heads = _dtype_code(k), _dtype_code(w_kr), cb.shape[0]
    args.q = _ptr(q)
    args.q_stride_b, args.q_stride_n, args.q_stride_h = q.stride(0), q.stride(1), q.stride(2)
    args.k = _ptr(k)
    args.k_stride_b, args.k_stride_n, args.k_stride_h = k.stride(0), k.stride(1), k.stride(2)
    args.w_qr, args.w_kr, args.codebook = _ptr(w_qr), _ptr(w_kr), _ptr(cb)
    args.indices = _ptr(indices)
    args.index_dtype = L.SSA_I64 if index_i64 else L.SSA_I32
    args.q_codes, args.k_codes, args.cand_counts = _ptr(q_codes), _ptr(k_codes), _ptr(cand_counts)
    return args


def _prep_weights(w_qr, w_kr, codebook, x_dtype=None):
    """Weights share one dtype: the input dtype or float32."""
    wd = w_kr.dtype
    if x_dtype is not None and wd not in (x_dtype, torch.float32):
        wd = torch.float32
    w_kr = w_kr.to(wd)
    w_qr = w_qr.to(wd).contiguous()
    w_kr = w_kr.contiguous()
    codebook = codebook.to(wd).contiguous()
    return w_qr, w_kr, codebook


def workspace(args: L.SsaRouteArgs, device) -> torch.Tensor:
    nbytes = L.lib().ssa_route_workspace_size(ctypes.byref(args))
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
# route
# ---------------------------------------------------------------------------
@torch.library.custom_op("ssa_b200::route", mutates_args=())
def route(q: torch.Tensor, k: torch.Tensor, w_qr: torch.Tensor, w_kr: torch.Tensor,
          codebook: torch.Tensor, a: int, b: int, top_k: int, causal: bool, temperature: float,
          q_offset: int, index_i64: bool) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = _require_cuda(q, k, w_qr, w_kr, codebook)
    q, k = _last_contig(q), _last_contig(k)
    w_qr, w_kr, codebook = _prep_weights(w_qr, w_kr, codebook, k.dtype)
    B, n_q, _, _ = q.shape
    _, n, h_kv, _ = k.shape
    indices = torch.empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32,
                          device=dev)
    q_codes = torch.empty((B, n_q, h_kv, a), dtype=torch.int32, device=dev)
    k_codes = torch.empty((B, n, h_kv, b), dtype=torch.int32, device=dev)
    counts = torch.empty((B, n_q, h_kv), dtype=torch.int32, device=dev)
    args = route_args(q, k, w_qr, w_kr, codebook, a, b, top_k, causal, temperature, q_offset,
                      indices, index_i64, q_codes, k_codes, counts)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_route", L.lib().ssa_route(ctypes.byref(args), ws.data_ptr(), ws.numel(),
                                               _stream(dev)))
        S.release(slot, "ssa_route", S.route_error)
    return indices, q_codes, k_codes, counts


@route.register_fake
def _route_fake(q, k, w_qr, w_kr, codebook, a, b, top_k, causal, temperature, q_offset, index_i64):
    B, n_q, _, _ = q.shape
    _, n, h_kv, _ = k.shape
    return (q.new_empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32),
            q.new_empty((B, n_q, h_kv, a), dtype=torch.int32),
            q.new_empty((B, n, h_kv, b), dtype=torch.int32),
            q.new_empty((B, n_q, h_kv), dtype=torch.int32))


# ---------------------------------------------------------------------------
# route_rope: rotate-half RoPE fused into the routing projection
# ---------------------------------------------------------------------------
def _rope_table(t: torch.Tensor, B: int, d: int) -> torch.Tensor:
    """``cos`` / ``sin`` as ``[1 or B, positions, d]`` with a contiguous last
    dimension; accepts ``[positions, d]``, ``[1|B, positions, d]`` and the
    head-broadcast forms ``[1|B, positions, 1, d]`` / ``[1|B, 1, positions, d]``."""
    if t.dim() == 4:
        if t.shape[2] == 1:
            t = t[:, :, 0]
        elif t.shape[1] == 1:
            t = t[:, 0]
        else:
            raise ValueError(f"RoPE table of shape {tuple(t.shape)} is not broadcast over heads")
    if t.dim() == 2:
        t = t.unsqueeze(0)
    if t.dim() != 3 or t.shape[-1] != d or t.shape[0] not in (1, B):
        raise ValueError(f"RoPE table of shape {tuple(t.shape)} does not fit batch {B}, head_dim {d}")
    return _last_contig(t)


@torch.library.custom_op("ssa_b200::route_rope", mutates_args=())
def route_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, w_qr: torch.Tensor,
               w_kr: torch.Tensor, codebook: torch.Tensor, a: int, b: int, top_k: int, causal: bool,
               temperature: float, q_offset: int, index_i64: bool
               ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """RoPE (rotate-half, ``x * cos + cat(-x2, x1) * sin`` in the dtype of q/k)
    applied to ``q [B, n_q, h_q, d]`` and ``k [B, n, h_kv, d]`` inside the
    routing projection, then stages 1-2 on the rotated rows.  Query row i uses
    table position ``q_offset + i``.  Returns ``(indices, q_codes, k_codes,
    cand_counts, q_rot, k_rot)``."""
    dev = _require_cuda(q, k, cos, sin, w_qr, w_kr, codebook)
    q, k = _last_contig(q), _last_contig(k)
    if cos.dtype != q.dtype or sin.dtype != q.dtype:
        raise ValueError("cos / sin must have the dtype of q and k")
    B, n_q, _, d = q.shape
    _, n, h_kv, _ = k.shape
    cos, sin = _rope_table(cos, B, d), _rope_table(sin, B, d)
    if cos.shape != sin.shape or cos.stride() != sin.stride():
        raise ValueError("cos and sin must have the same shape and strides")
    if cos.shape[1] < max(n, q_offset + n_q):
        raise ValueError(f"RoPE tables cover {cos.shape[1]} positions, {max(n, q_offset + n_q)} needed")
    w_qr, w_kr, codebook = _prep_weights(w_qr, w_kr, codebook, k.dtype)
    indices = torch.empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32,
                          device=dev)
    q_codes = torch.empty((B, n_q, h_kv, a), dtype=torch.int32, device=dev)
    k_codes = torch.empty((B, n, h_kv, b), dtype=torch.int32, device=dev)
    counts = torch.empty((B, n_q, h_kv), dtype=torch.int32, device=dev)
    q_rot, k_rot = torch.empty_like(q, memory_format=torch.contiguous_format), \
        torch.empty_like(k, memory_format=torch.contiguous_format)
    args = route_args(q, k, w_qr, w_kr, codebook, a, b, top_k, causal, temperature, q_offset,
                      indices, index_i64, q_codes, k_codes, counts)
    rope = L.SsaRopeArgs()
    rope.cos, rope.sin = cos.data_ptr(), sin.data_ptr()
    rope.table_stride_b = cos.stride(0) if cos.shape[0] > 1 else 0
    rope.table_stride_n = cos.stride(1)
    rope.q_out = q_rot.data_ptr()
    rope.q_out_stride_b, rope.q_out_stride_n, rope.q_out_stride_h = q_rot.stride(0), q_rot.stride(1), q_rot.stride(2)
    rope.k_out = k_rot.data_ptr()
    rope.k_out_stride_b, rope.k_out_stride_n, rope.k_out_stride_h = k_rot.stride(0), k_rot.stride(1), k_rot.stride(2)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_route_rope", L.lib().ssa_route_rope(ctypes.byref(args), ctypes.byref(rope), ws.data_ptr(),
                                                         ws.numel(), _stream(dev)))
        S.release(slot, "ssa_route_rope", S.route_error)
    return indices, q_codes, k_codes, counts, q_rot, k_rot


@route_rope.register_fake
def _route_rope_fake(q, k, cos, sin, w_qr, w_kr, codebook, a, b, top_k, causal, temperature, q_offset, index_i64):
    B, n_q, _, _ = q.shape
    _, n, h_kv, _ = k.shape
    return (q.new_empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32),
            q.new_empty((B, n_q, h_kv, a), dtype=torch.int32),
            q.new_empty((B, n, h_kv, b), dtype=torch.int32),
            q.new_empty((B, n_q, h_kv), dtype=torch.int32),
            torch.empty_like(q, memory_format=torch.contiguous_format),
            torch.empty_like(k, memory_format=torch.contiguous_format))


# ---------------------------------------------------------------------------
# route_with_key_codes
# ---------------------------------------------------------------------------
@torch.library.custom_op("ssa_b200::route_with_key_codes", mutates_args=())
def route_with_key_codes(q: torch.Tensor, k: torch.Tensor, k_codes: torch.Tensor, w_qr: torch.Tensor,
                         w_kr: torch.Tensor, codebook: torch.Tensor, a: int, top_k: int, causal: bool,
                         temperature: float, q_offset: int, index_i64: bool) -> torch.Tensor:
    """Stages 1-2 for the query rows ``q [B, n_q, h_q, d]`` at sequence positions
    ``q_offset ..`` against all keys ``k [B, n, h_kv, d]``, whose codes
    ``k_codes [B, n, h_kv, b]`` (from :func:`code_assign`) are given."""
    dev = _require_cuda(q, k, k_codes, w_qr, w_kr, codebook)
    q, k = _last_contig(q), _last_contig(k)
    kc = k_codes.to(torch.int32).contiguous()
    w_qr, w_kr, codebook = _prep_weights(w_qr, w_kr, codebook, k.dtype)
    B, n_q, _, _ = q.shape
    _, n, h_kv, _ = k.shape
    if tuple(kc.shape[:3]) != (B, n, h_kv):
        raise ValueError(f"k_codes shape {tuple(kc.shape)} does not match k {tuple(k.shape)}")
    indices = torch.empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32,
                          device=dev)
    args = route_args(q, k, w_qr, w_kr, codebook, a, kc.shape[-1], top_k, causal, temperature,
                      q_offset, indices, index_i64, None, kc, None)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_route_with_key_codes",
                L.lib().ssa_route_with_key_codes(ctypes.byref(args), ws.data_ptr(), ws.numel(),
                                                 _stream(dev)))
        S.release(slot, "ssa_route_with_key_codes", S.route_error)
    return indices


@route_with_key_codes.register_fake
def _route_with_key_codes_fake(q, k, k_codes, w_qr, w_kr, codebook, a, top_k, causal, temperature,
                               q_offset, index_i64):
    B, n_q, _, _ = q.shape
    h_kv = k.shape[2]
    return q.new_empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32)


@torch.library.custom_op("ssa_b200::route_with_index", mutates_args=())
def route_with_index(q: torch.Tensor, k: torch.Tensor, k_codes: torch.Tensor, bucket_ptr: torch.Tensor,
                     bucket_keys: torch.Tensor, w_qr: torch.Tensor, w_kr: torch.Tensor, codebook: torch.Tensor,
                     a: int, top_k: int, causal: bool, temperature: float, q_offset: int,
                     index_i64: bool) -> torch.Tensor:
    """:func:`route_with_key_codes` with the code->key index of ``k_codes``
    given too (``bucket_ptr``, ``bucket_keys`` from :func:`build_index`), so
    that several query blocks of one sequence share one index build."""
    dev = _require_cuda(q, k, k_codes, bucket_ptr, bucket_keys, w_qr, w_kr, codebook)
    q, k = _last_contig(q), _last_contig(k)
    kc = k_codes.to(torch.int32).contiguous()
    ptr = bucket_ptr.to(torch.int32).contiguous()
    keys = bucket_keys.to(torch.int32).contiguous()
    w_qr, w_kr, codebook = _prep_weights(w_qr, w_kr, codebook, k.dtype)
    B, n_q, _, _ = q.shape
    _, n, h_kv, _ = k.shape
    if tuple(kc.shape[:3]) != (B, n, h_kv):
        raise ValueError(f"k_codes shape {tuple(kc.shape)} does not match k {tuple(k.shape)}")
    n_codes = codebook.shape[-2]
    if ptr.numel() != B * h_kv * (n_codes + 1) or keys.numel() != B * h_kv * n * kc.shape[-1]:
        raise ValueError("bucket_ptr / bucket_keys do not match k_codes and the codebook")
    indices = torch.empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32,
                          device=dev)
    args = route_args(q, k, w_qr, w_kr, codebook, a, kc.shape[-1], top_k, causal, temperature,
                      q_offset, indices, index_i64, None, kc, None)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_route_with_index",
                L.lib().ssa_route_with_index(ctypes.byref(args), ptr.data_ptr(), keys.data_ptr(), ws.data_ptr(),
                                             ws.numel(), _stream(dev)))
        S.release(slot, "ssa_route_with_index", S.route_error)
    return indices


@route_with_index.register_fake
def _route_with_index_fake(q, k, k_codes, bucket_ptr, bucket_keys, w_qr, w_kr, codebook, a, top_k, causal,
                           temperature, q_offset, index_i64):
    B, n_q, _, _ = q.shape
    return q.new_empty((B, n_q, k.shape[2], top_k), dtype=torch.int64 if index_i64 else torch.int32)


# ---------------------------------------------------------------------------
# query rows in segments (several blocks of one sequence in one call)
# ---------------------------------------------------------------------------
def segments_struct(blocks) -> L.SsaQuerySegments:
    """``blocks``: ``[(position, rows), ...]`` in ascending positions."""
    if not 1 <= len(blocks) <= L.SSA_MAX_SEGMENTS:
        raise ValueError(f"{len(blocks)} query segments: 1..{L.SSA_MAX_SEGMENTS} supported")
    s = L.SsaQuerySegments()
    s.count = len(blocks)
    for i, (pos, rows) in enumerate(blocks):
        s.positions[i], s.rows[i] = int(pos), int(rows)
    return s


def route_with_index_segments(q, k, k_codes, bucket_ptr, bucket_keys, w_qr, w_kr, codebook, a, top_k, causal,
                              temperature, blocks, index_i64=False):
    """:func:`route_with_index` for query rows ``q [B, n_q, h_q, d]`` that are
    several runs of positions ``blocks = [(position, rows), ...]`` (ascending),
    in one call: the GPU of a sequence shard routes all its blocks at once."""
    dev = _require_cuda(q, k, k_codes, bucket_ptr, bucket_keys, w_qr, w_kr, codebook)
    q, k = _last_contig(q), _last_contig(k)
    kc = k_codes.to(torch.int32).contiguous()
    ptr = bucket_ptr.to(torch.int32).contiguous()
    keys = bucket_keys.to(torch.int32).contiguous()
    w_qr, w_kr, codebook = _prep_weights(w_qr, w_kr, codebook, k.dtype)
    B, n_q, _, _ = q.shape
    _, n, h_kv, _ = k.shape
    indices = torch.empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32, device=dev)
    args = route_args(q, k, w_qr, w_kr, codebook, a, kc.shape[-1], top_k, causal, temperature, 0, indices,
                      index_i64, None, kc, None)
    segs = segments_struct(blocks)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_route_with_index_segments",
                L.lib().ssa_route_with_index_segments(ctypes.byref(args), ctypes.byref(segs), ptr.data_ptr(),
                                                      keys.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev)))
        S.release(slot, "ssa_route_with_index_segments", S.route_error)
    return indices


def query_codes(q, w_qr, codebook, a, h_kv, temperature=1.0):
    """The query half of stage 1: ``q [B, n_q, h_q, d]`` -> the ``a`` codes
    ``[B, n_q, h_kv, a]`` int32 of every query group (``ssa_query_codes``).
    Needs no keys: the first half of :func:`route_with_index_segments` for a
    GPU whose keys are still being gathered."""
    dev = _require_cuda(q, w_qr, codebook)
    q = _last_contig(q)
    w_qr, _, codebook = _prep_weights(w_qr, w_qr, codebook, q.dtype)
    B, n_q, h_q, _ = q.shape
    if h_q % h_kv:
        raise ValueError(f"num_q_heads ({h_q}) must be a multiple of num_kv_heads ({h_kv})")
    q_codes = torch.empty((B, n_q, h_kv, a), dtype=torch.int32, device=dev)
    if B == 0 or n_q == 0:
        return q_codes
    # the key fields describe the query rows themselves (checked, not read)
    args = route_args(q, q[:, :, :h_kv], w_qr, w_qr, codebook, a, 1, 1, False, temperature, 0,
                      q_codes=q_codes)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_query_codes", L.lib().ssa_query_codes(ctypes.byref(args), ws.data_ptr(), ws.numel(),
                                                           _stream(dev)))
        S.release(slot, "ssa_query_codes", S.route_error)
    return q_codes


def select_candidates_segments(q, k, q_codes, k_codes, bucket_ptr, bucket_keys, top_k, causal, blocks,
                               index_i64=False):
    """The second half of :func:`route_with_index_segments`: stage 2 for the
    query rows ``q`` in runs of positions ``blocks`` from their codes
    ``q_codes`` (:func:`query_codes`), the keys' codes and their index."""
    dev = _require_cuda(q, k, q_codes, k_codes, bucket_ptr, bucket_keys)
    q, k = _last_contig(q), _last_contig(k)
    qc = q_codes.to(torch.int32).contiguous()
    kc = k_codes.to(torch.int32).contiguous()
    ptr = bucket_ptr.to(torch.int32).contiguous()
    keys = bucket_keys.to(torch.int32).contiguous()
    B, n_q, _, d = q.shape
    # routing weights are not read by stage 2; these placeholders carry N_c
    w = torch.empty((4, d), dtype=k.dtype, device=dev)
    cb = torch.empty((1, ptr.shape[-1] - 1, 4), dtype=k.dtype, device=dev)
    indices = torch.empty((B, n_q, k.shape[2], top_k), dtype=torch.int64 if index_i64 else torch.int32,
                          device=dev)
    args = route_args(q, k, w, w, cb, qc.shape[-1], kc.shape[-1], top_k, causal, 1.0, 0, indices, index_i64,
                      qc, kc, None)
    segs = segments_struct(blocks)
    slot = S.acquire(dev)
    args.status = slot.ptr if slot is not None else None
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_select_candidates_segments",
                L.lib().ssa_select_candidates_segments(ctypes.byref(args), ctypes.byref(segs), ptr.data_ptr(),
                                                       keys.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev)))
        S.release(slot, "ssa_select_candidates_segments", S.route_error)
    return indices


def sparse_attn_segments(q, k, v, indices, scale, causal, blocks):
    """:func:`sparse_attn` for query rows in runs of positions ``blocks =
    [(position, rows), ...]`` (ascending), in one launch."""
    dev = _require_cuda(q, k, v, indices)
    q, k, v, indices = _last_contig(q), _last_contig(k), _last_contig(v), _last_contig(indices)
    out = torch.empty(q.shape, dtype=q.dtype, device=dev)
    segs = segments_struct(blocks)
    slot = S.acquire(dev)
    args = attn_args(q, k, v, indices, out, scale, causal, 0, slot.ptr if slot is not None else None)
    with torch.cuda.device(dev):
        L.check("ssa_sparse_attn_segments",
                L.lib().ssa_sparse_attn_segments(ctypes.byref(args), ctypes.byref(segs), _stream(dev)))
        S.release(slot, "sparse_exact_attention", S.attn_error)
    return out


# ---------------------------------------------------------------------------
# code_assign
# ---------------------------------------------------------------------------
@torch.library.custom_op("ssa_b200::code_assign", mutates_args=())
def code_assign(k: torch.Tensor, w_kr: torch.Tensor, codebook: torch.Tensor, b: int,
                temperature: float) -> torch.Tensor:
    dev = _require_cuda(k, w_kr, codebook)
    k = _last_contig(k)
    _, w_kr, codebook = _prep_weights(w_kr, w_kr, codebook, k.dtype)
    B, n, h_kv, _ = k.shape
    k_codes = torch.empty((B, n, h_kv, b), dtype=torch.int32, device=dev)
    # q-side fields mirror k (unused by ssa_code_assign)
    args = route_args(k, k, w_kr, w_kr, codebook, 1, b, 1, False, temperature, 0,
                      k_codes=k_codes)
    args.n_q = 0
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_code_assign", L.lib().ssa_code_assign(ctypes.byref(args), ws.data_ptr(),
                                                           ws.numel(), _stream(dev)))
    return k_codes


@code_assign.register_fake
def _code_assign_fake(k, w_kr, codebook, b, temperature):
    B, n, h_kv, _ = k.shape
    return k.new_empty((B, n, h_kv, b), dtype=torch.int32)


# ---------------------------------------------------------------------------
# sparse_attn
# ---------------------------------------------------------------------------
def attn_args(q, k, v, indices, out, scale, causal, q_offset, status=None):
    B, n_q, h_q, d = q.shape
    _, n, h_kv, _ = k.shape
    args = L.SsaAttnArgs()
    args.batch, args.n_q, args.n, args.q_offset = B, n_q, n, q_offset
    args.h_q, args.h_kv, args.d, args.top_k = h_q, h_kv, d, indices.shape[-1]
    args.causal, args.scale, args.dtype = int(bool(causal)), float(scale), _dtype_code(q)
    args.q = q.data_ptr()
    args.q_stride_b, args.q_stride_n, args.q_stride_h = q.stride(0), q.stride(1), q.stride(2)
    args.k = k.data_ptr()
    args.k_stride_b, args.k_stride_n, args.k_stride_h = k.stride(0), k.stride(1), k.stride(2)
    args.v = v.data_ptr()
    args.v_stride_b, args.v_stride_n, args.v_stride_h = v.stride(0), v.stride(1), v.stride(2)
    args.indices = indices.data_ptr()
    args.index_dtype = L.SSA_I64 if indices.dtype == torch.int64 else L.SSA_I32
    args.idx_stride_b, args.idx_stride_n, args.idx_stride_h = (indices.stride(0), indices.stride(1),
                                                                indices.stride(2))
    args.out = out.data_ptr()
    args.out_stride_b, args.out_stride_n, args.out_stride_h = out.stride(0), out.stride(1), out.stride(2)
    # the status word: a device address (an int) or a one-element int32 tensor
    args.status = status if status is None or isinstance(status, int) else status.data_ptr()
    return args


@torch.library.custom_op("ssa_b200::sparse_attn", mutates_args=())
def sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                scale: float, causal: bool, q_offset: int) -> torch.Tensor:
    dev = _require_cuda(q, k, v, indices)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError(f"q, k, v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    if indices.dtype not in (torch.int64, torch.int32):
        raise TypeError(f"indices must be int64 or int32, got {indices.dtype}")
    q, k, v, indices = _last_contig(q), _last_contig(k), _last_contig(v), _last_contig(indices)
    out = torch.empty(q.shape, dtype=q.dtype, device=dev)
    slot = S.acquire(dev)
    args = attn_args(q, k, v, indices, out, scale, causal, q_offset, slot.ptr if slot is not None else None)
    with torch.cuda.device(dev):
        L.check("ssa_sparse_attn", L.lib().ssa_sparse_attn(ctypes.byref(args), _stream(dev)))
        S.release(slot, "sparse_exact_attention", S.attn_error)
    return out


@sparse_attn.register_fake
def _sparse_attn_fake(q, k, v, indices, scale, causal, q_offset):
    return torch.empty_like(q)


@torch.library.custom_op("ssa_b200::sparse_attn_backward", mutates_args=())
def sparse_attn_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor,
                         out: torch.Tensor, d_out: torch.Tensor, scale: float, causal: bool,
                         q_offset: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients ``(dq, dk, dv)`` of :func:`sparse_attn` at output gradient
    ``d_out`` (``out`` is the forward output).  dK and dV are accumulated in
    fp32 with atomic adds, so their last bits depend on the order of the adds."""
    dev = _require_cuda(q, k, v, indices, out, d_out)
    q = q.contiguous()
    k, v, indices = _last_contig(k), _last_contig(v), _last_contig(indices)
    out = out.contiguous()
    d_out = d_out.to(out.dtype).contiguous()
    B, n, h_kv, d = k.shape
    dq = torch.empty_like(q)
    dk = torch.empty((B, n, h_kv, d), dtype=torch.float32, device=dev)
    dv = torch.empty((B, n, h_kv, d), dtype=torch.float32, device=dev)
    slot = S.acquire(dev)
    args = attn_args(q, k, v, indices, out, scale, causal, q_offset, slot.ptr if slot is not None else None)
    with torch.cuda.device(dev):
        L.check("ssa_sparse_attn_backward",
                L.lib().ssa_sparse_attn_backward(ctypes.byref(args), d_out.data_ptr(), dq.data_ptr(),
                                                 dk.data_ptr(), dv.data_ptr(), _stream(dev)))
        S.release(slot, "sparse_exact_attention backward", S.attn_error)
    return dq, dk.to(k.dtype), dv.to(v.dtype)


@sparse_attn_backward.register_fake
def _sparse_attn_backward_fake(q, k, v, indices, out, d_out, scale, causal, q_offset):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


def _sparse_attn_setup(ctx, inputs, output):
    q, k, v, indices, scale, causal, q_offset = inputs
    ctx.save_for_backward(q, k, v, indices, output)
    ctx.scale, ctx.causal, ctx.q_offset = scale, causal, q_offset


def _sparse_attn_grad(ctx, d_out):
    q, k, v, indices, out = ctx.saved_tensors
    dq, dk, dv = sparse_attn_backward(q, k, v, indices, out, d_out, ctx.scale, ctx.causal, ctx.q_offset)
    return dq, dk, dv, None, None, None, None


sparse_attn.register_autograd(_sparse_attn_grad, setup_context=_sparse_attn_setup)


# ---------------------------------------------------------------------------
# test hooks (not custom ops): bit-exact parity of the selection stages
# ---------------------------------------------------------------------------
def select_from_scores(scores: torch.Tensor, kk: int) -> torch.Tensor:
    """Top-``kk`` of each row of fp32 ``scores [rows, n_cols]`` (score desc, index asc)."""
    dev = _require_cuda(scores)
    s = scores.to(torch.float32).contiguous()
    rows, n_cols = s.reshape(-1, s.shape[-1]).shape
    out = torch.empty((rows, kk), dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        L.check("ssa_select_from_scores",
                L.lib().ssa_select_from_scores(s.data_ptr(), rows, n_cols, kk, out.data_ptr(),
                                               _stream(dev)))
    return out.reshape(*scores.shape[:-1], kk)


def index_args(B: int, n: int, h_kv: int, b: int, n_codes: int, placeholder: torch.Tensor) -> L.SsaRouteArgs:
    """:class:`SsaRouteArgs` for the index-only calls (``ssa_build_index`` and
    ``ssa_build_index_noalloc``), which read the sizes and nothing else: the
    pointers the argument check wants set all name ``placeholder`` (any
    16-byte-aligned device buffer; it is never read) and the strides are 0."""
    args = L.SsaRouteArgs()
    args.batch, args.n, args.n_q, args.q_offset = B, n, 0, 0
    args.h_q, args.h_kv, args.d, args.d_s = h_kv, h_kv, 8, 4
    args.n_codes, args.a, args.b, args.top_k = n_codes, 1, b, 1
    args.causal, args.temperature = 0, 1.0
    args.dtype, args.w_dtype, args.codebook_heads = L.SSA_F32, L.SSA_F32, 1
    p = placeholder.data_ptr()
    args.q = args.k = args.w_qr = args.w_kr = args.codebook = p
    return args


def build_index(k_codes: torch.Tensor, n_codes: int, h_q: int = 1):
    """Inverted index of ``k_codes [B, n, h_kv, b]`` -> ``(bucket_ptr, bucket_keys)``."""
    dev = _require_cuda(k_codes)
    kc = k_codes.to(torch.int32).contiguous()
    B, n, h_kv, b = kc.shape
    ptr = torch.empty((B, h_kv, n_codes + 1), dtype=torch.int32, device=dev)
    args = index_args(B, n, h_kv, b, n_codes, ptr)
    keys = torch.empty((B, h_kv, n * b), dtype=torch.int32, device=dev)
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_build_index", L.lib().ssa_build_index(ctypes.byref(args), kc.data_ptr(),
                                                           ptr.data_ptr(), keys.data_ptr(),
                                                           ws.data_ptr(), ws.numel(), _stream(dev)))
    return ptr, keys


def select_candidates(q, k, q_codes, k_codes, n_codes, top_k, causal=True, q_offset=0,
                      index_i64=True):
    """Stage 2 alone from given codes -> ``(indices, cand_counts)``."""
    dev = _require_cuda(q, k, q_codes, k_codes)
    q, k = _last_contig(q), _last_contig(k)
    qc = q_codes.to(torch.int32).contiguous()
    kc = k_codes.to(torch.int32).contiguous()
    B, n_q, h_q, d = q.shape
    _, n, h_kv, _ = k.shape
    w = torch.empty((4, d), dtype=k.dtype, device=dev)
    cb = torch.empty((1, n_codes, 4), dtype=k.dtype, device=dev)
    idx = torch.empty((B, n_q, h_kv, top_k), dtype=torch.int64 if index_i64 else torch.int32,
                      device=dev)
    counts = torch.empty((B, n_q, h_kv), dtype=torch.int32, device=dev)
    args = route_args(q, k, w, w, cb, qc.shape[-1], kc.shape[-1], top_k, causal, 1.0, q_offset,
                      idx, index_i64, qc, kc, counts)
    ws = workspace(args, dev)
    with torch.cuda.device(dev):
        L.check("ssa_select_candidates",
                L.lib().ssa_select_candidates(ctypes.byref(args), ws.data_ptr(), ws.numel(),
                                              _stream(dev)))
    return idx, counts
