"""The allocation-free index build: ssa_build_index_noalloc.

Some callers cannot allocate device memory -- code that runs inside a CUDA
stream capture, under a runtime that owns all device memory, or in a loop
that must never allocate.  ssa_build_index_noalloc serves them: it takes no
workspace and keeps its scratch in an array built into the library.

This file checks, through the C ABI, that it returns exactly what
ssa_build_index (which uses a caller-provided workspace) returns, on two calls
in a row with different inputs -- the second call reuses the same built-in
scratch, so stale contents from the first call must not leak into it.  It also
checks that a size needing more than the built-in scratch is refused.  The
file name sorts last so that a run stopping at the first failure has run
every other test already.
"""

import ctypes

import numpy as np
import pytest
import torch

from ssa_b200 import _lib as L
from ssa_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _args(B, n, h_kv, b, n_codes):
    # the index build takes no K: the args carry sizes, and the pointers the
    # argument check wants set name one small placeholder that is never read
    placeholder = torch.empty(4, dtype=torch.int32, device=DEV)
    return ops.index_args(B, n, h_kv, b, n_codes, placeholder), placeholder


def _codes(seed, B, n, h_kv, b, n_codes):
    rng = np.random.default_rng(seed)
    kc = rng.integers(0, n_codes, size=(B, n, h_kv, b), dtype=np.int32)
    return torch.from_numpy(kc).to(DEV)


def _with_workspace(kc, n_codes):
    B, n, h_kv, b = kc.shape
    args, keep = _args(B, n, h_kv, b, n_codes)
    ptr = torch.empty((B, h_kv, n_codes + 1), dtype=torch.int32, device=DEV)
    keys = torch.empty((B, h_kv, n * b), dtype=torch.int32, device=DEV)
    ws = ops.workspace(args, DEV)
    rc = L.lib().ssa_build_index(ctypes.byref(args), kc.data_ptr(), ptr.data_ptr(), keys.data_ptr(),
                                 ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    L.check("ssa_build_index", rc)
    return ptr, keys


def _no_alloc(kc, n_codes):
    B, n, h_kv, b = kc.shape
    args, keep = _args(B, n, h_kv, b, n_codes)
    # poison the outputs: every element must be written by the call
    ptr = torch.full((B, h_kv, n_codes + 1), -7, dtype=torch.int32, device=DEV)
    keys = torch.full((B, h_kv, n * b), -7, dtype=torch.int32, device=DEV)
    rc = L.lib().ssa_build_index_noalloc(ctypes.byref(args), kc.data_ptr(), ptr.data_ptr(), keys.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    L.check("ssa_build_index_noalloc", rc)
    return ptr, keys


def test_no_alloc_index_matches_workspace_version_twice():
    # two different problems back to back on the same built-in scratch
    cases = [(11, 2, 5000, 3, 4, 4096), (12, 1, 20000, 8, 4, 1024)]
    for seed, B, n, h_kv, b, n_codes in cases:
        kc = _codes(seed, B, n, h_kv, b, n_codes)
        ref_ptr, ref_keys = _with_workspace(kc, n_codes)
        got_ptr, got_keys = _no_alloc(kc, n_codes)
        torch.cuda.synchronize()
        assert torch.equal(got_ptr, ref_ptr)
        assert torch.equal(got_keys, ref_keys)


def test_no_alloc_index_rejects_sizes_beyond_its_scratch():
    # B*h_kv*n_codes*tiles counts: 8*8192*128 words = 32 MiB > 16 MiB
    args, keep = _args(1, 131072, 8, 4, 8192)
    buf = torch.empty(16, dtype=torch.int32, device=DEV)
    rc = L.lib().ssa_build_index_noalloc(ctypes.byref(args), buf.data_ptr(), buf.data_ptr(), buf.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 2                                          # SSA_ERR_UNSUPPORTED
    assert b"scratch" in L.lib().ssa_last_error()
