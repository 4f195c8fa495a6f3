"""C-ABI checks that need no GPU: the library loads, exports every function
declared in include/ssa_b200.h, the ctypes mirrors have the C layout, and
argument errors come back as status codes before anything is launched."""

import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from ssa_b200 import _lib as L
from ssa_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ssa_b200.h")


@pytest.fixture(scope="module")
def lib():
    build()
    return L.lib()


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\**\s+\**(ssa_[a-z_0-9]+)\s*\(", text, re.M)))


def test_header_declares_expected_entry_points():
    names = declared_functions()
    for n in ["ssa_route", "ssa_route_workspace_size", "ssa_code_assign", "ssa_sparse_attn",
              "ssa_select_from_scores", "ssa_build_index", "ssa_select_candidates",
              "ssa_status_str", "ssa_last_error"]:
        assert n in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (ssa_\w+)", out))
    assert set(declared_functions()) <= exported
    assert set(L.SIGNATURES) == set(declared_functions())


def _c_layout(struct: str, fields):
    src = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
           f'printf("%zu\\n", sizeof({struct}));']
    src += [f'printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    src += ["return 0;}"]
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        open(c, "w").write("\n".join(src))
        subprocess.run(["gcc", "-std=c99", c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], capture_output=True, text=True).stdout.split()]
    return vals[0], vals[1:]


@pytest.mark.parametrize("cls,name", [(L.SsaRouteArgs, "SsaRouteArgs"), (L.SsaAttnArgs, "SsaAttnArgs"),
                                      (L.SsaRopeArgs, "SsaRopeArgs"),
                                      (L.SsaDecodeIndex, "SsaDecodeIndex"),
                                      (L.SsaQuerySegments, "SsaQuerySegments")])
def test_ctypes_structs_match_c_layout(cls, name):
    fields = [f for f, _ in cls._fields_]
    size, offsets = _c_layout(name, fields)
    assert ctypes.sizeof(cls) == size
    assert [getattr(cls, f).offset for f in fields] == offsets


def _route_args(**over):
    a = L.SsaRouteArgs()
    vals = dict(batch=1, n=64, n_q=64, q_offset=0, h_q=8, h_kv=2, d=64, d_s=32, n_codes=128, a=8, b=4,
                top_k=16, causal=1, temperature=1.0, dtype=L.SSA_BF16, w_dtype=L.SSA_F32,
                codebook_heads=2, q=0x1000, q_stride_b=64 * 8 * 64, q_stride_n=8 * 64, q_stride_h=64,
                k=0x2000, k_stride_b=64 * 2 * 64, k_stride_n=2 * 64, k_stride_h=64, w_qr=0x3000,
                w_kr=0x4000, codebook=0x5000, indices=0x6000, index_dtype=L.SSA_I64)
    vals.update(over)
    for kk, v in vals.items():
        setattr(a, kk, v)
    return a


def test_workspace_size_is_host_only_and_positive(lib):
    a = _route_args()
    ws = lib.ssa_route_workspace_size(ctypes.byref(a))
    assert ws > 64 * 2 * (32 * 4)
    assert lib.ssa_route_workspace_size(None) == 0


def test_workspace_grows_with_the_query_units(lib):
    # every (query, KV head) unit needs its routed vector (d_s fp32), its a
    # codes and one slot in each of the three overflow lists of the re-score
    # tiers; regions are 256-byte aligned, hence the slack
    small = lib.ssa_route_workspace_size(ctypes.byref(_route_args(n=4096, n_q=1024)))
    large = lib.ssa_route_workspace_size(ctypes.byref(_route_args(n=4096, n_q=4096)))
    units = (4096 - 1024) * 2
    per_unit = 32 * 4 + 8 * 4 + 3 * 4
    assert large - small >= units * per_unit - 32 * 256


@pytest.mark.parametrize("over,code", [
    (dict(h_q=7), 1),                 # not a multiple of h_kv
    (dict(d=60), 2),                  # head_dim not a multiple of 8
    (dict(d_s=24), 2),                # unsupported route_dim
    (dict(a=40), 2),                  # codes_per_query > 32
    (dict(top_k=0), 1),
    (dict(n=0), 1),
    (dict(temperature=0.0), 1),
    (dict(codebook_heads=3), 1),
    (dict(k=0x2004), 4),              # misaligned k
    (dict(q_offset=10), 1),           # q_offset + n_q > n
    (dict(top_k=20000, n=20000, n_q=20000), 2),  # min(k, n) above the shared-memory capacity
    # 2^31 (sequence, KV head, query) units: the re-score numbers units with 32-bit ints
    (dict(batch=1 << 14, h_kv=8, n=1 << 14, n_q=1 << 14, top_k=16), 2),
])
def test_route_argument_errors(lib, over, code):
    a = _route_args(**over)
    ws = ctypes.create_string_buffer(16)
    rc = lib.ssa_route(ctypes.byref(a), ctypes.addressof(ws), 16, None)
    assert rc == code, lib.ssa_last_error()
    assert lib.ssa_last_error()


def test_route_rejects_small_workspace(lib):
    a = _route_args()
    rc = lib.ssa_route(ctypes.byref(a), None, 0, None)
    assert rc == 3
    assert b"workspace" in lib.ssa_last_error()


def test_attn_argument_errors(lib):
    a = L.SsaAttnArgs()
    a.batch, a.n_q, a.n, a.h_q, a.h_kv, a.d, a.top_k, a.scale, a.dtype = 1, 8, 8, 34, 2, 64, 4, 8.0, 1
    a.q = a.k = a.v = a.indices = a.out = 0x1000
    assert lib.ssa_sparse_attn(ctypes.byref(a), None) == 2          # group 17 > 16
    a.h_q = 8
    a.d = 12
    assert lib.ssa_sparse_attn(ctypes.byref(a), None) == 2
    a.d = 64
    a.batch, a.n_q, a.n = 1 << 14, 1 << 16, 1 << 16          # 2^31 (sequence, head, query) units
    assert lib.ssa_sparse_attn(ctypes.byref(a), None) == 2
    assert b"2^31" in lib.ssa_last_error()
    assert lib.ssa_sparse_attn(None, None) == 1


def test_select_from_scores_argument_errors(lib):
    assert lib.ssa_select_from_scores(None, 1, 8, 4, None, None) == 1
    assert lib.ssa_select_from_scores(0x1000, 1, 8, 40, 0x2000, None) == 2


def test_status_strings(lib):
    for code in range(7):
        assert lib.ssa_status_str(code)


def _rope_args(**over):
    r = L.SsaRopeArgs()
    vals = dict(cos=0x7000, sin=0x8000, table_stride_b=0, table_stride_n=64,
                q_out=0x9000, q_out_stride_b=64 * 8 * 64, q_out_stride_n=8 * 64, q_out_stride_h=64,
                k_out=0xa000, k_out_stride_b=64 * 2 * 64, k_out_stride_n=2 * 64, k_out_stride_h=64)
    vals.update(over)
    for kk, v in vals.items():
        setattr(r, kk, v)
    return r


@pytest.mark.parametrize("route_over,rope_over,code", [
    ({"dtype": L.SSA_F32}, {}, 2),          # fp32 q/k: no tensor-core projection
    ({"d": 96, "q_stride_h": 96, "k_stride_h": 96}, {}, 2),   # head_dim not 64/128
    ({}, {"cos": 0}, 1),
    ({}, {"k_out": 0}, 1),
    ({}, {"table_stride_n": 32}, 1),       # rows of the table overlap
    ({}, {"q_out": 0x9008}, 4),
    ({}, {"table_stride_n": 68}, 4),
])
def test_route_rope_argument_errors(lib, route_over, rope_over, code):
    a = _route_args(**route_over)
    r = _rope_args(**rope_over)
    assert lib.ssa_route_rope(ctypes.byref(a), ctypes.byref(r), None, 0, None) == code


def test_route_rope_null_rope_is_an_argument_error(lib):
    a = _route_args()
    assert lib.ssa_route_rope(ctypes.byref(a), None, None, 0, None) == 1


def _segments(rows, positions):
    s = L.SsaQuerySegments()
    s.count = len(rows)
    for i, (r, p) in enumerate(zip(rows, positions)):
        s.rows[i], s.positions[i] = r, p
    return s


@pytest.mark.parametrize("rows,positions,ok", [
    ([32, 32], [0, 32], True),
    ([16, 48], [0, 16], True),
    ([32, 32], [32, 0], False),          # positions must ascend
    ([32, 32], [0, 16], False),          # runs overlap
    ([32, 31], [0, 32], False),          # rows do not add up to n_q
    ([32, 32], [0, 40], False),          # the last run ends past n
    ([8] * 9, list(range(0, 72, 8)), False),   # more than SSA_MAX_SEGMENTS
])
def test_segment_argument_checks(lib, rows, positions, ok):
    """Segment checks run before any launch; valid segments then fail only on
    the (deliberately missing) workspace, never as argument errors."""
    a = _route_args(k_codes=0x7000)
    s = _segments(rows[:8], positions[:8])
    if len(rows) > 8:
        s.count = len(rows)
    rc = lib.ssa_route_with_index_segments(ctypes.byref(a), ctypes.byref(s), 0x8000, 0x9000, None, 0, None)
    assert rc == (3 if ok else 1), lib.ssa_last_error()
    a.q_codes = 0xa000
    rc = lib.ssa_select_candidates_segments(ctypes.byref(a), ctypes.byref(s), 0x8000, 0x9000, None, 0, None)
    assert rc == (3 if ok else 1), lib.ssa_last_error()
    at = L.SsaAttnArgs()
    at.batch, at.n_q, at.n, at.h_q, at.h_kv, at.d, at.top_k, at.scale, at.dtype = 1, 64, 64, 8, 2, 64, 4, 8.0, 1
    at.q = at.k = at.v = at.indices = at.out = 0x1000
    if not ok:
        assert lib.ssa_sparse_attn_segments(ctypes.byref(at), ctypes.byref(s), None) == 1
