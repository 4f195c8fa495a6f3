"""SSA forward benchmark on B200: tokens/s of one forward pass of the hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--n 32768]

Workload (BASELINE config 3 at its quoted point): batch 1, n = 32768,
h_q = 32, h_kv = 8, d = 128, d_s = 32, N_c = 4096, a = 16, b = 4, k = 256,
causal, bf16, planted-cluster synthetic inputs (seeded).  One step = the
whole forward: the router (routing projection, codebook scoring with top-a /
top-b, inverted index, candidate re-score + top-k) and the sparse exact
attention over the selected keys.

* ``value``: whole-job tokens/s with inputs resident in HBM, timed on the
  device (CUDA events, barrier + synchronize on both sides, max over ranks).
  Inputs (q 268 MB + k 67 MB + v 67 MB) exceed the 126 MB L2; no flush.
* ``e2e``: the same forward through the public drop-in API
  (``CodebookRouter`` -> ``sparse_exact_attention``) from pinned HOST
  buffers: host->device copies of q/k/v and the device->host copy of the
  output are inside the timed region.
* ``roofline``: the sparse-attention kernel (the largest share of the step):
  its compulsory HBM bytes (q, out, K, V, indices once) per launch / its
  CUDA-event duration against the measured HBM copy bandwidth, the ncu DRAM
  traffic of a launch beside them, and in ``l2`` the logical bytes (every
  gathered K/V row) against the L2 read peak measured in the same run -- the
  gathers are served from L2, so that fraction is the one that binds.
  ``roofline_stages``: stage 1 (codebook scoring, tensor) and stage 2
  (index + re-score + top-k, DRAM and L2 as above).
* ``parity``: the timed step's own codes, indices and output against the CPU
  oracle on a sample (one KV head, ~580 query rows), outside the timed region.
* ``cpu_baseline``: the reference algorithm (CPU oracle port, O(n^2) dense
  re-score as the reference computes it) on a bounded sample, rank 0 only.
* ``config4``: config 4 (one n = 131072 sequence split by queries over the
  ranks, NCCL all-gathers of K, V and key codes) timed in the same process
  group: its strong-scaling curve over the driver's N = 1, 2, 4, 8 runs.

Multi-GPU (torchrun, one process per GPU): for the headline each rank runs its
own independent sequence (batch x KV-head units need no exchange) -> weak
scaling.  ``--impl reference`` times the reference's CPU algorithm (oracle
port) on the host cores instead.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SSA fwd tokens/s per GPU (n=32k, k=256, bf16) and % of HBM/tensor roofline"
UNIT = "tokens/s"
# kernels of libssa_sm100a.so launched per step (config 3, bf16): route = codebook normalise,
# codebook tensor-core image, 2x projection, 2x tcgen05 code scoring, key index (count, 3x
# scan, scatter, entry codes), bucket-major re-score (group-mean rows, query index: count,
# 3x scan, scatter; bucket lengths, bucket tiles, per-query selection), the walking
# re-score's second and third tiers and the general overflow pass (for the units the
# bucket path had no room for); attention = 1.  (The cudaMemsetAsync calls that clear the
# counters are not kernels and are not counted.)
LAUNCHES_PER_STEP = 25
# DRAM bytes (read + write) of one sparse-attention launch at config 3, n = 32768,
# measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum, one pass on this
# workload; profiles/sparse_attn_mma_config3.txt).  Other n scale by the query rows.
ATTN_DRAM_BYTES_N32768 = 920.29e6
# DRAM bytes of stage 2 (ssa_select_candidates: the code->key index with its
# entry codes, then the bucket-major re-score: group-mean rows, code->query
# index, bucket lengths, bucket tiles, selection) per call at n = 32768: the sum
# of the ncu dram__bytes_read.sum + dram__bytes_write.sum of its kernels in one
# route call of the bench's workload (profiles/rescore_bucket_config3.txt); the
# candidate segments (written by the tiles, read by the selection) are 1.1 GB of it.
RESCORE_DRAM_BYTES_N32768 = 2233e6


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--n", type=int, default=32768)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-config4", action="store_true",
                   help="skip the config-4 (query-split n=131072) record of the default run")
    p.add_argument("--workload", default="config3", choices=["config3", "config4", "config5", "decode"],
                   help="config3: one sequence per GPU (the headline); config4: one n=131072 "
                        "sequence split by queries over the GPUs (strong scaling); config5: a Qwen-style "
                        "28-layer decoder stack with SSA attention, one batch per GPU")
    p.add_argument("--layers", type=int, default=28, help="config5: decoder layers")
    p.add_argument("--batch", type=int, default=4, help="config5: sequences per GPU")
    p.add_argument("--folds", type=int, default=4,
                   help="config4: zig-zag passes; each rank holds 2 * folds blocks of the sequence")
    p.add_argument("--kv-after-qcodes", action="store_true",
                   help="config4: issue the K and V all-gathers after the query codes")
    p.add_argument("--v-after-qcodes", action="store_true",
                   help="config4: issue the V all-gather after the query codes (K with the codes)")
    p.add_argument("--timeline", action="store_true",
                   help="config4: after the timed steps, one step with CUDA events between its phases")
    p.add_argument("--emulate", default=None, metavar="RANK/WORLD",
                   help="config4, one GPU: time the work of rank RANK of WORLD with the gathered tensors "
                        "already in place (no exchange), by phase and by kernel")
    return p.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.flush()
        rows = []
        with open(self.f.name) as fh:
            for line in fh:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        # every sample taken while the timed region ran (no filtering)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_mhz_min": min(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows),
                "interval_ms": 100}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's forward (torch-CPU port), bounded sample
# ---------------------------------------------------------------------------
def cpu_sample(t_cpu, shape, heads=1, rows=None):
    """Times the reference forward on the host for ``heads`` KV heads: key
    codes of all n keys, then the last ``rows`` query rows (all rows by
    default): query codes, the dense re-score over all n keys with the
    candidate mask and top-k, and the gathered attention.  Returns (tokens/s
    for the whole step, extrapolated over the rows and the h_kv heads,
    seconds, description)."""
    import torch
    from oracle import ssa_port_torch as P

    q, k, v, w_qr, w_kr, cb = t_cpu
    n, g = shape.n, shape.h_q // shape.h_kv
    rows = n if rows is None else min(rows, n)
    i0 = n - rows
    P.attention(q[:8, :g].contiguous(), k[:, 0].contiguous(), v[:, 0].contiguous(),
                torch.zeros((8, 4), dtype=torch.int64))            # thread-pool warm-up
    t0 = time.perf_counter()
    key_s = 0.0
    for h in range(heads):
        qh = q[i0:, h * g:(h + 1) * g].contiguous()
        kh, vh = k[:, h].contiguous(), v[:, h].contiguous()
        ta = time.perf_counter()
        kc = P.key_codes(kh, w_kr, cb[h], shape.b)
        key_s += time.perf_counter() - ta
        qc = P.query_codes(qh, w_qr, cb[h], shape.a)
        idx = P.select(qh, kh, qc, kc, shape.n_codes, shape.top_k, i0, True)
        P.attention(qh, kh, vh, idx, i0, True)
    elapsed = time.perf_counter() - t0
    per_head = (key_s + (elapsed - key_s) * n / rows) / heads
    seconds = per_head * shape.h_kv
    sample = (f"{heads} of {shape.h_kv} KV heads: key codes of all {n} keys + "
              + (f"all {n} query rows" if rows == n else f"the last {rows} query rows")
              + f" (query codes, dense re-score over {n} keys with candidate mask, top-{shape.top_k},"
              f" gathered attention), fp32 torch CPU port of the reference forward, extrapolated to "
              f"{shape.h_kv} heads" + ("" if rows == n else f" and {n} rows"))
    return n / seconds, elapsed, sample


def cpu_inputs(shape, seed):
    import torch
    from ssa_b200 import workloads as W

    t = W.make_inputs(shape, seed=seed, dtype=torch.bfloat16, device="cpu")
    f = lambda x: (x[0] if x.dim() == 4 else x).float().contiguous()
    return f(t["q"]), f(t["k"]), f(t["v"]), t["w_qr"].float(), t["w_kr"].float(), t["codebook"].float()


def bench_config(shape, world):
    """The ``config`` dict of the config-3 line; both arms print the same one."""
    mb = shape.n * (shape.h_q + 2 * shape.h_kv) * shape.d * 2 / 1e6
    return {"workload": f"config3 (op-level sweep at n={shape.n})", **shape.asdict(),
            "per_rank": "one independent sequence per GPU",
            "l2": f"inputs {mb:.0f} MB {'>' if mb > 126 else '<'} 126 MB L2, no flush",
            "parallelism": f"batch-units x{world}"}


def run_reference(args):
    """The reference's CPU algorithm (oracle port) on the host cores.  Each
    step is a bounded sample of the config-3 forward: one KV head, key codes
    of all n keys, then the last n/4 query rows (query codes, dense masked
    re-score over all n keys, top-k, gathered attention).  ``ms_per_step`` is
    the measured time of that sampled step; ``value`` is the tokens/s of the
    full forward extrapolated from it (the key codes once per head, the rows
    by n / rows, the h_kv heads by h_kv)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return 0
    import torch
    from ssa_b200 import workloads as W

    shape = W.Shape(**{**W.CONFIG3.asdict(), "n": args.n})
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    t_cpu = cpu_inputs(shape, args.seed)
    rows = max(1, shape.n // 4)
    vals, secs = [], []
    t0 = time.perf_counter()
    for it in range(args.warmup + args.steps):
        v, s, sample = cpu_sample(t_cpu, shape, heads=1, rows=rows)
        if it >= args.warmup:
            vals.append(v)
            secs.append(s)
    wall = time.perf_counter() - t0
    value = statistics.median(vals)
    ms_step = 1e3 * statistics.median(secs)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded: Q/K ~ N(0,1), 5% planted keys around 64 centroids, V ~ N(0,1))",
            "config": bench_config(shape, world),
            "work_per_step": {"kv_heads": 1, "of_kv_heads": shape.h_kv, "keys_coded": shape.n,
                              "query_rows": rows, "of_query_rows": shape.n},
            "ms_per_full_forward_extrapolated": 1e3 * shape.n / value,
            "wall_s": wall,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample, "sample_seconds": statistics.median(secs)},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def measure_l2_read_peak(dev, reps=50):
    """L2 read bandwidth (outside the timed region): ``ssa_l2_read_probe``
    (16-byte L2-only loads over the whole GPU) on 16 / 32 / 48 MiB buffers
    that stay in the 126 MB L2, one launch of ``reps`` passes each, timed with
    CUDA events; the best of the sizes.  The denominator of the ``l2``
    fractions below."""
    import torch
    from ssa_b200 import _lib as L

    lib = L.lib()
    sink = torch.zeros(1, dtype=torch.int64, device=dev)
    st = torch.cuda.current_stream(dev)
    best = 0.0
    for mib in (16, 32, 48):
        x = torch.ones(mib * 2 ** 20 // 4, device=dev)
        for _ in range(2):
            L.check("ssa_l2_read_probe", lib.ssa_l2_read_probe(x.data_ptr(), x.numel() * 4, 2, sink.data_ptr(),
                                                               st.cuda_stream))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        L.check("ssa_l2_read_probe", lib.ssa_l2_read_probe(x.data_ptr(), x.numel() * 4, reps, sink.data_ptr(),
                                                           st.cuda_stream))
        e1.record(st)
        torch.cuda.synchronize(dev)
        best = max(best, mib * 2 ** 20 * reps / (e0.elapsed_time(e1) / 1e3) / 1e9)
        del x
    return best


def bench_parity(t, shape, idx, q_codes, k_codes, out, head=1, n_rows=512, seed=7):
    """Sampled parity of the measured step's own outputs against the CPU
    oracle (outside the timed region): one KV head, ``n_rows`` query rows
    spread over the sequence plus the last 64.  Reports the fraction of key
    and query code rows equal to the oracle's, the candidate-set overlap with
    the oracle's selection and the relative L2 error of the attention output
    against the float64 oracle on the GPU's own selection (
    >= 0.999, >= 0.999, <= 2e-3)."""
    import numpy as np
    import torch
    from oracle import ssa_oracle as O

    t0 = time.perf_counter()
    n, g = shape.n, shape.h_q // shape.h_kv
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([rng.choice(n, size=n_rows, replace=False), np.arange(n - 64, n)]))
    rt = torch.from_numpy(rows).to(idx.device)
    f64 = lambda x: x.double().cpu().numpy()
    q_rows = f64(t["q"][0, rt, head * g:(head + 1) * g])
    k_h, v_h = f64(t["k"][0, :, head]), f64(t["v"][0, :, head])
    kc, qc, ref_idx = O.route_rows_one_head(q_rows, rows, k_h, f64(t["w_qr"]), f64(t["w_kr"]),
                                            f64(t["codebook"][head]), shape.a, shape.b, shape.top_k, causal=True)
    same = lambda a, b: float((np.sort(a, -1) == np.sort(b, -1)).all(-1).mean())
    gi = idx[0, rt, head].long().cpu().numpy()
    sa, sb = np.sort(gi, 1), np.sort(ref_idx, 1)
    overlap = sum(np.intersect1d(x, y).size for x, y in zip(sa, sb)) / gi.size
    ref_out = O.sparse_attention(q_rows, k_h[:, None], v_h[:, None], gi[:, None], causal=True, positions=rows)
    got = f64(out[0, rt, head * g:(head + 1) * g])
    rel = float(np.linalg.norm(got - ref_out) / np.linalg.norm(ref_out))
    return {"kv_head": head, "query_rows": int(rows.size), "key_code_rows_equal": same(k_codes[0, :, head].cpu().numpy(), kc),
            "query_code_rows_equal": same(q_codes[0, rt, head].cpu().numpy(), qc),
            "candidate_overlap": overlap, "output_rel_l2_err": rel,
            "oracle": "oracle/ssa_oracle.py route_rows_one_head + sparse_attention (float64)",
            "seconds": time.perf_counter() - t0}
def stage_rooflines(lib, rargs, q_codes, k_codes, cand, shape, ws, sptr, stream, hbm, tflops, peak_kind,
                    l2_peak, reps=10):
    """Rooflines of the two router stages, each timed with CUDA events in its
    own loop after the timed region (the C ABI launches a stage's kernels in
    one call, so they cannot be bracketed inside ssa_route):
      stage 1 (keys): ssa_code_assign -- codebook scoring of the n*h_kv keys on
        tensor cores, 2*n*h_kv*N_c*d_s useful flops (plus the projection);
      stage 2: ssa_select_candidates -- code->key index, then the bucket-major
        re-score: group-mean rows, code->query index, bucket tiles writing each
        query's candidate segment, per-query top-k.  Algorithmic bytes: the q
        rows once (g*d*2 a unit), the group-mean hi/lo rows written once and read
        once per code (2*d*2*(1 + a)), every key row staged once per code it holds
        (b*d*2 a key), 8 bytes a candidate written and read back (16*C, C the
        unique candidates of the unit from the route's cand_counts), k*4 out."""
    import torch
    from ssa_b200 import _lib as L

    n, hkv, g, d = shape.n, shape.h_kv, shape.h_q // shape.h_kv, shape.d
    c_sum = int(cand.sum().item())
    units = n * hkv
    s2_bytes = (16 * c_sum + units * (g * d * 2 + 2 * d * 2 * (1 + shape.a) + shape.top_k * 4)
                + n * hkv * shape.b * d * 2)
    # the same stage as the per-query formulation defines its work: every
    # candidate's key row, id and codes gathered once per query that reaches it
    walk_bytes = c_sum * (4 + 16 + 2 * d) + units * (g * d * 2 + shape.top_k * 4)
    s1_flops = 2.0 * n * hkv * shape.n_codes * shape.d_s

    def timed(fn):
        for _ in range(2):
            fn()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    kc = torch.empty_like(k_codes)
    a1 = L.SsaRouteArgs.from_buffer_copy(rargs)
    a1.k_codes = kc.data_ptr()
    a1.n_q = 0
    t1 = timed(lambda: L.check("ssa_code_assign",
                               lib.ssa_code_assign(ctypes.byref(a1), ws.data_ptr(), ws.numel(), sptr)))
    a2 = L.SsaRouteArgs.from_buffer_copy(rargs)
    t2 = timed(lambda: L.check("ssa_select_candidates",
                               lib.ssa_select_candidates(ctypes.byref(a2), ws.data_ptr(), ws.numel(), sptr)))
    f1 = s1_flops / (t1 / 1e3) / 1e12
    dram2 = RESCORE_DRAM_BYTES_N32768 * n / 32768
    return {
        "stage1_keys": {"call": "ssa_code_assign", "bound": "tensor", "achieved": f1, "peak": tflops,
                        "unit": "TFLOP/s", "frac": f1 / tflops, "peak_kind": peak_kind,
                        "algorithmic_flops": s1_flops, "ms": t1},
        # stage 2 against the DRAM copy peak (ncu DRAM bytes of the stage's
        # kernels) and the measured L2 read peak (algorithmic bytes); both
        # fractions are low: its kernels are bound by dependent loads and
        # instruction issue (selection sort, radix select), not by bandwidth
        "stage2": {"call": "ssa_select_candidates", "bound": "hbm", "unit": "GB/s", "ms": t2,
                   "achieved": dram2 / (t2 / 1e3) / 1e9, "peak": hbm, "peak_kind": peak_kind,
                   "frac": dram2 / (t2 / 1e3) / 1e9 / hbm, "traffic": dram2,
                   "l2": {"achieved": s2_bytes / (t2 / 1e3) / 1e9, "peak": l2_peak,
                          "frac": s2_bytes / (t2 / 1e3) / 1e9 / l2_peak, "bytes": s2_bytes},
                   "logical_bytes": s2_bytes, "mean_unique_candidates": c_sum / units,
                   "per_query_equivalent": {
                       "bytes": walk_bytes, "achieved": walk_bytes / (t2 / 1e3) / 1e9, "unit": "GB/s",
                       "frac_of_hbm": walk_bytes / (t2 / 1e3) / 1e9 / hbm,
                       "note": "bytes a per-query re-score gathers (the survey's K3 work); the "
                               "bucket-major path moves logical_bytes instead"}},
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    from ssa_b200 import _lib as L
    from ssa_b200 import ops
    from ssa_b200 import workloads as W
    import ssa_b200 as ssa

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1 or not args.no_config4:
        init_group(dev, world, 180)

    shape = W.Shape(**{**W.CONFIG3.asdict(), "n": args.n})
    t = W.make_inputs(shape, seed=args.seed + rank, dtype=torch.bfloat16, device=dev)
    q, k, v = t["q"], t["k"], t["v"]
    n, hq, hkv, d, kk = shape.n, shape.h_q, shape.h_kv, shape.d, shape.top_k
    lib = L.lib()

    # preallocated outputs + workspace; calls go straight through the C ABI
    idx = torch.empty((1, n, hkv, kk), dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    q_codes = torch.empty((1, n, hkv, shape.a), dtype=torch.int32, device=dev)
    k_codes = torch.empty((1, n, hkv, shape.b), dtype=torch.int32, device=dev)
    cand = torch.empty((1, n, hkv), dtype=torch.int32, device=dev)
    w_qr, w_kr, cb = t["w_qr"].contiguous(), t["w_kr"].contiguous(), t["codebook"].contiguous()
    rargs = ops.route_args(q, k, w_qr, w_kr, cb, shape.a, shape.b, kk, True, 1.0, 0, idx, False,
                           q_codes, k_codes, cand)
    ws = ops.workspace(rargs, dev)
    aargs = ops.attn_args(q, k, v, idx, out, math.sqrt(d), True, 0)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        L.check("ssa_route", lib.ssa_route(ctypes.byref(rargs), ws.data_ptr(), ws.numel(), sptr))
        if ev is not None:
            ev[1].record(stream)
        L.check("ssa_sparse_attn", lib.ssa_sparse_attn(ctypes.byref(aargs), sptr))
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for s in range(args.steps):
        step(evs[s])
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    route_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    attn_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    if world > 1:
        tt = torch.tensor([total_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = float(tt.item())
    ms_step = total_ms / args.steps
    value = world * n / (ms_step / 1e3)
    in_mb = sum(x.numel() * x.element_size() for x in (q, k, v)) / 1e6

    # roofline of the sparse-attention kernel (one launch per step).  Its
    # algorithmic HBM bytes are the compulsory ones (q and out once, K and V
    # once, the int32 indices once); its k gathered K/V rows per (query, head)
    # -- the logical bytes -- come from L2 (head-major order keeps a head's K/V
    # resident), so the L2 read rate against the measured L2 read peak is the
    # fraction that binds it.
    hbm, tflops, peak_kind = load_peaks()
    l2_peak = measure_l2_read_peak(dev)
    units = n * hkv
    attn_logical = units * kk * (2 * d * 2) + 2 * n * hq * d * 2 + units * kk * 4
    attn_compulsory = 2 * n * hq * d * 2 + 2 * n * hkv * d * 2 + units * kk * 4
    attn_s = attn_ms / 1e3
    traffic = ATTN_DRAM_BYTES_N32768 * n / 32768
    roof = {"kernel": "sparse_attn_mma_kernel", "bound": "hbm", "unit": "GB/s",
            "achieved": attn_compulsory / attn_s / 1e9, "peak": hbm, "peak_kind": peak_kind,
            "frac": attn_compulsory / attn_s / 1e9 / hbm,
            "traffic": traffic,
            "traffic_note": "ncu DRAM read + write bytes per launch at n=32768"
                            + ("" if n == 32768 else ", scaled by n"),
            "algorithmic_bytes_per_launch": attn_compulsory,
            "dram_frac": traffic / attn_s / 1e9 / hbm,
            "l2": {"achieved": attn_logical / attn_s / 1e9, "peak": l2_peak, "unit": "GB/s",
                   "frac": attn_logical / attn_s / 1e9 / l2_peak, "bytes": attn_logical,
                   "peak_kind": "measured in this run: ssa_l2_read_probe (L2-only 16-byte reads of a 16-48 MiB buffer)"},
            "binding": "l2 (k gathered K/V rows per query and head, served from L2)",
            "logical_bytes_per_launch": attn_logical, "launch_ms": attn_ms, "router_ms": route_ms}
    # parity of the timed steps' own outputs, before anything rewrites them
    parity = bench_parity(t, shape, idx, q_codes, k_codes, out) if rank == 0 else None
    stages = stage_rooflines(lib, rargs, q_codes, k_codes, cand, shape, ws, sptr, stream, hbm, tflops,
                             peak_kind, l2_peak)

    # e2e through the public API from pinned host buffers, with the API's
    # default device-status checking (read back lazily, no host stall).  Every
    # step copies its q/k/v in (host -> device) and its output back (device ->
    # host); the copies run on two copy streams so that step s+1's inputs and
    # step s-1's output move while step s computes (double-buffered inputs).
    e2e = None
    if not args.no_e2e:
        router = ssa.CodebookRouter(head_dim=d, route_dim=shape.d_s, num_kv_heads=hkv,
                                    num_codebook=shape.n_codes, codes_per_key=shape.b,
                                    codes_per_query=shape.a, top_k=kk).to(dev)
        with torch.no_grad():
            router.W_qr.weight.copy_(w_qr)
            router.W_kr.weight.copy_(w_kr)
            router.codebook.copy_(cb)
        host_in = [x[0].cpu().pin_memory() for x in (q, k, v)]
        host_out = [torch.empty(host_in[0].shape, dtype=host_in[0].dtype).pin_memory() for _ in range(2)]
        dev_in = [[torch.empty_like(x, device=dev) for x in host_in] for _ in range(2)]
        h2d_stream = torch.cuda.Stream(dev)
        d2h_stream = torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event() for _ in range(2)]
        in_free = [torch.cuda.Event() for _ in range(2)]

        def h2d(sidx):
            b = sidx % 2
            h2d_stream.wait_event(in_free[b])
            with torch.cuda.stream(h2d_stream):
                for dst, src in zip(dev_in[b], host_in):
                    dst.copy_(src, non_blocking=True)
            in_ready[b].record(h2d_stream)

        def run(steps):
            h2d(0)
            for sidx in range(steps):
                if sidx + 1 < steps:
                    h2d(sidx + 1)
                b = sidx % 2
                stream.wait_event(in_ready[b])
                dq, dk, dv = dev_in[b]
                with torch.no_grad():
                    ind = router(dq, dk, causal=True)
                    o = ssa.sparse_exact_attention(dq, dk, dv, ind, is_causal=True)
                in_free[b].record(stream)
                done = torch.cuda.Event()
                done.record(stream)
                d2h_stream.wait_event(done)
                with torch.cuda.stream(d2h_stream):
                    host_out[b].copy_(o, non_blocking=True)
                o.record_stream(d2h_stream)
            stream.wait_stream(d2h_stream)

        run(max(3, args.warmup))
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d_stream.wait_event(e0)
        run(args.steps)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ssa.check_errors(dev)                     # the steps' device status words: all clear
        e_ms = e0.elapsed_time(e1)
        if world > 1:
            tt = torch.tensor([e_ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = float(tt.item())
        e2e = {"value": world * n / (e_ms / args.steps / 1e3), "unit": UNIT,
               "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in host_in),
               "d2h_bytes_per_step": host_out[0].numel() * host_out[0].element_size(),
               "ms_per_step": e_ms / args.steps,
               "api": "CodebookRouter.forward + sparse_exact_attention (default SSA_CHECKED: lazy status)",
               "copies": "pinned host buffers; h2d of step s+1 and d2h of step s overlap step s's compute"}
        del host_in, host_out, dev_in
        torch.cuda.empty_cache()

    # config 4 (one n = 131072 sequence split by queries over the ranks, NCCL
    # all-gathers) in the same process group: the driver's N = 1..8 runs of
    # this script then record its strong-scaling curve too
    c4 = None
    if not args.no_config4:
        del q, k, v, t, out, idx, ws
        torch.cuda.empty_cache()
        c4 = config4_timing(args, dev, world, rank, steps=max(3, min(args.steps, 10)), warmup=3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cores = os.cpu_count() or 1
        torch.set_num_threads(cores)
        cv, cs, sample = cpu_sample(cpu_inputs(shape, args.seed), shape, heads=2)
        cpu = {"value": cv, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
               "sample_seconds": cs}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded: Q/K ~ N(0,1), 5% planted keys around 64 centroids, V ~ N(0,1))",
                "config": bench_config(shape, world),
                "roofline": roof, "roofline_stages": stages, "parity": parity, "cpu_baseline": cpu,
                "e2e": e2e, "clocks": clk, "gpu_launches": LAUNCHES_PER_STEP * args.steps,
                "config4": c4}
        print(json.dumps(line), flush=True)
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    return 0


def init_group(dev, world, timeout_s):
    """One NCCL process group over the ranks torchrun started (a 1-rank group
    on 127.0.0.1 for a plain ``python bench.py``)."""
    import datetime
    import socket

    import torch.distributed as dist

    if world == 1 and "MASTER_ADDR" not in os.environ:
        with socket.socket() as so:
            so.bind(("127.0.0.1", 0))
            port = so.getsockname()[1]
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="1")
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=dev)


def config4_timing(args, dev, world, rank, steps, warmup):
    """Config 4: one long sequence (n = 131072, N_c = 8192, k = 512, bf16,
    N(0,1) inputs) split by queries over the ranks of the current process group
    (ssa_b200.shard: zig-zag blocks, all-gather of K, V and key codes, routing
    with the gathered codes, attention).  Total work is fixed: strong scaling.
    Device-timed (CUDA events, barrier + synchronize on both sides, max over
    ranks).  Returns the record rank 0 prints."""
    import torch
    import torch.distributed as dist

    import ssa_b200 as ssa
    from ssa_b200 import shard
    from ssa_b200 import workloads as W

    n = W.CONFIG4.n if args.workload != "config4" or args.n == 32768 else args.n
    shape = W.Shape(**{**W.CONFIG4.asdict(), "n": n})
    t = W.make_inputs(shape, seed=args.seed, dtype=torch.bfloat16, device=dev, planted=False,
                      generate_on_device=True)
    router = ssa.CodebookRouter(head_dim=shape.d, route_dim=shape.d_s, num_kv_heads=shape.h_kv,
                                num_codebook=shape.n_codes, codes_per_key=shape.b, codes_per_query=shape.a,
                                top_k=shape.top_k).to(dev)
    with torch.no_grad():
        router.W_qr.weight.copy_(t["w_qr"])
        router.W_kr.weight.copy_(t["w_kr"])
        router.codebook.copy_(t["codebook"])
    folds = args.folds
    ql, kl, vl = (shard.local_rows(t[x], world, rank, folds=folds) for x in ("q", "k", "v"))
    del t
    torch.cuda.empty_cache()
    stream = torch.cuda.current_stream(dev)

    def step(marks=None):
        with torch.no_grad():
            return shard.sharded_forward(router, ql, kl, vl, causal=True, folds=folds,
                                         kv_after_query_codes=args.kv_after_qcodes,
                                         v_after_query_codes=args.v_after_qcodes, marks=marks)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(dev)
    ssa.check_errors(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dist.barrier()
    clk = clocks.stop()
    ssa.check_errors(dev)
    tt = torch.tensor([e0.elapsed_time(e1)], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms_step = float(tt.item()) / steps
    timeline = None
    if getattr(args, "timeline", False):
        # one more step, outside the timed region, with events between its
        # phases; every rank's durations, gathered on rank 0
        marks = []
        step(marks)
        torch.cuda.synchronize(dev)
        phases = [name for name, _ in marks[1:]]
        mine = [round(marks[i][1].elapsed_time(marks[i + 1][1]), 3) for i in range(len(marks) - 1)]
        every = [None] * world
        dist.all_gather_object(every, mine)
        timeline = {"phases": phases, "ms_by_rank": every,
                    "max_ms": [max(r[i] for r in every) for i in range(len(phases))]}
    del ql, kl, vl
    torch.cuda.empty_cache()
    return {"metric": "SSA fwd tokens/s, one n=131072 sequence split over the GPUs (k=512, bf16)",
            "value": n / (ms_step / 1e3), "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (seeded on device: Q/K/V ~ N(0,1))",
            "config": {"workload": "config4 (long single sequence, query-split)", **shape.asdict(),
                       "parallelism": f"query-split x{world} ({2 * folds} zig-zag blocks per rank routed and "
                                      "attended in one call each, NCCL all-gather of K, V, codes)",
                       "l2": "inputs 1.6 GB > 126 MB L2, no flush"},
            "clocks": clk, **({"timeline": timeline} if timeline else {})}


def config4_emulation(args, dev):
    """``--workload config4 --emulate R/W`` on one GPU: the compute of rank
    ``R`` of a ``W``-rank config-4 forward, with the gathered K, V and key
    codes already in place, so that the exchange and its interference with
    the kernels are left out.  The phases are those of
    ``ssa_b200.shard.sharded_forward`` without the collectives: key codes of
    the rank's own keys, the rank's query codes, the code->key index of all
    ``n`` keys, one candidate-selection call and one attention call over the
    rank's blocks.  Reports the CUDA-event time per step and per phase, and
    the device time per kernel (torch.profiler over the same steps)."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    import ssa_b200 as ssa
    from ssa_b200 import ops, shard
    from ssa_b200 import workloads as W

    rank, world = (int(x) for x in args.emulate.split("/"))
    shape = W.CONFIG4
    n = shape.n
    folds = args.folds
    t = W.make_inputs(shape, seed=args.seed, dtype=torch.bfloat16, device=dev, planted=False,
                      generate_on_device=True)
    router = ssa.CodebookRouter(head_dim=shape.d, route_dim=shape.d_s, num_kv_heads=shape.h_kv,
                                num_codebook=shape.n_codes, codes_per_key=shape.b, codes_per_query=shape.a,
                                top_k=shape.top_k).to(dev)
    with torch.no_grad():
        router.W_qr.weight.copy_(t["w_qr"])
        router.W_kr.weight.copy_(t["w_kr"])
        router.codebook.copy_(t["codebook"])
    k_full, v_full = t["k"], t["v"]
    ql, kl = (shard.local_rows(t[x], world, rank, folds=folds) for x in ("q", "k"))
    del t
    blocks = shard.zigzag_blocks(n, world, rank, folds)
    codes_full = router.key_codes(k_full)
    stream = torch.cuda.current_stream(dev)

    def step(marks=None):
        def mark(name):
            if marks is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record(stream)
                marks.append((name, ev))

        with torch.no_grad():
            mark("start")
            router.key_codes(kl)
            mark("key codes")
            q_codes = ops.query_codes(ql, router.W_qr.weight, router.codebook, router.codes_per_query,
                                      router.num_kv_heads, float(router.temperature))
            mark("query codes")
            index = router.key_index(codes_full)
            mark("index")
            idx = ops.select_candidates_segments(ql, k_full, q_codes, codes_full, index[0], index[1],
                                                 router.top_k, True, blocks)
            mark("candidates")
            out = ops.sparse_attn_segments(ql, k_full, v_full, idx, math.sqrt(shape.d), True, blocks)
            mark("attention")
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ssa.check_errors(dev)
    clocks = ClockSampler(dev.index)
    clocks.start()
    marks_all = []
    for _ in range(args.steps):
        marks = []
        step(marks)
        marks_all.append(marks)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    ssa.check_errors(dev)
    phases = [name for name, _ in marks_all[0][1:]]
    per_phase = [sum(m[i][1].elapsed_time(m[i + 1][1]) for m in marks_all) / args.steps
                 for i in range(len(phases))]
    ms_step = sum(m[0][1].elapsed_time(m[-1][1]) for m in marks_all) / args.steps
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            step()
        torch.cuda.synchronize(dev)
    kernels = {}
    for e in prof.key_averages():
        us = getattr(e, "self_device_time_total", None)
        if us is None:
            us = e.self_cuda_time_total
        if us > 0:
            kernels[e.key] = round(us / 1e3 / args.steps, 3)
    kernels = dict(sorted(kernels.items(), key=lambda kv: -kv[1]))
    print(json.dumps({
        "metric": "config-4 rank work emulated on one GPU (no exchange), ms per step",
        "emulated_rank": rank, "emulated_world": world, "folds": folds, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
        "phases": phases, "phase_ms": [round(x, 3) for x in per_phase],
        "kernel_ms_per_step": kernels, "clocks": clk,
        "config": {"workload": "config4", **shape.asdict(), "blocks": blocks},
        "data": "synthetic (seeded on device: Q/K/V ~ N(0,1))"}), flush=True)
    return 0


def run_config4(args):
    """``--workload config4``: the config-4 record alone, as its own line."""
    import torch
    import torch.distributed as dist

    if args.emulate:
        torch.cuda.set_device(0)
        return config4_emulation(args, torch.device("cuda", 0))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_group(dev, world, 180)
    rec = config4_timing(args, dev, world, rank, args.steps, args.warmup)
    if rank == 0:
        print(json.dumps({**rec, "vs_baseline": None, "roofline": None, "cpu_baseline": None, "e2e": None}),
              flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_config5(args):
    """Config 5: forward of a Qwen-style decoder stack (28 layers, d_model
    3584, 28 query / 4 KV heads of 128 -> GQA group 7, SwiGLU 18944, RMSNorm,
    RoPE base 1e6, q/k/v biases, vocab 152064, random-init bf16 weights) with
    every attention layer replaced by SSA (d_s 32, N_c 4096, b 4, a 16,
    k 256): per layer RoPE + CodebookRouter.route in one call
    (CodebookRouter.route_rope) and the sparse attention on the sm_100a
    kernels, the dense projections and the MLP as cuBLAS GEMMs.  Inputs are
    batch x n token ids uniform over the vocabulary; the LM head is not run
    (its bf16 logits alone would take 20 GB); the step is the stack's
    forward up to the final norm.  Each GPU runs its own batch (replicas)."""
    import datetime

    import torch
    import torch.nn.functional as F

    import ssa_b200 as ssa
    from ssa_b200 import ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    H, hq, hkv, hd, inter, vocab = 3584, 28, 4, 128, 18944, 152064
    B = args.batch
    n = args.n if args.n != 32768 else 16384
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(args.seed)

    def w(*shape, scale):
        return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * scale).to(dt)

    layers = []
    for _ in range(args.layers):
        r = ssa.CodebookRouter(head_dim=hd, route_dim=32, num_kv_heads=hkv, num_codebook=4096, codes_per_key=4,
                               codes_per_query=16, top_k=256).to(dev)
        layers.append(dict(
            ln1=torch.ones(H, device=dev, dtype=dt), ln2=torch.ones(H, device=dev, dtype=dt),
            wq=w(hq * hd, H, scale=H ** -0.5), bq=w(hq * hd, scale=0.02),
            wk=w(hkv * hd, H, scale=H ** -0.5), bk=w(hkv * hd, scale=0.02),
            wv=w(hkv * hd, H, scale=H ** -0.5), bv=w(hkv * hd, scale=0.02),
            wo=w(H, hq * hd, scale=(hq * hd) ** -0.5),
            wg=w(inter, H, scale=H ** -0.5), wu=w(inter, H, scale=H ** -0.5), wd=w(H, inter, scale=inter ** -0.5),
            router=r))
    emb = w(vocab, H, scale=0.02)
    ln_f = torch.ones(H, device=dev, dtype=dt)
    ids = torch.randint(0, vocab, (B, n), generator=g, device=dev)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd))
    ang = torch.arange(n, device=dev, dtype=torch.float32)[:, None] * inv_freq[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1).to(dt)[None, :, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1).to(dt)[None, :, None, :]

    def rms(x, wt):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dt) * wt

    attn_ms = [0.0]

    def forward(time_attn=False):
        x = emb[ids]
        for L in layers:
            h = rms(x, L["ln1"])
            q = F.linear(h, L["wq"], L["bq"]).view(B, n, hq, hd)
            k = F.linear(h, L["wk"], L["bk"]).view(B, n, hkv, hd)
            v = F.linear(h, L["wv"], L["bv"]).view(B, n, hkv, hd)
            if time_attn:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
            # position-indexed rotate-half RoPE, applied by the routing projection
            idx, q, k = L["router"].route_rope(q, k, cos, sin, causal=True, index_dtype=torch.int32)
            o = ops.sparse_attn(q, k, v, idx, hd ** 0.5, True, 0)
            if time_attn:
                e1.record()
                torch.cuda.synchronize(dev)
                attn_ms[0] += e0.elapsed_time(e1)
            x = x + F.linear(o.reshape(B, n, hq * hd), L["wo"])
            h = rms(x, L["ln2"])
            x = x + F.linear(F.silu(F.linear(h, L["wg"])) * F.linear(h, L["wu"]), L["wd"])
        return rms(x, ln_f)

    with torch.no_grad():
        for _ in range(args.warmup):
            forward()
        torch.cuda.synchronize(dev)
        clocks = ClockSampler(local)
        clocks.start()
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        stream = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            out = forward()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        clk = clocks.stop()
        total = e0.elapsed_time(e1)
        if dist:
            tt = torch.tensor([total], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            total = float(tt.item())
        forward(time_attn=True)                       # one more step, synchronised per layer: SSA share
        finite = bool(torch.isfinite(out).all())
    ms_step = total / args.steps
    if rank == 0:
        line = {"metric": "Qwen-style stack forward tokens/s with SSA attention (bf16)",
                "value": world * B * n / (ms_step / 1e3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init weights, token ids uniform over the vocabulary)",
                "config": {"workload": "config5 (Qwen-style decoder stack, SSA in every layer)",
                           "layers": args.layers, "d_model": H, "h_q": hq, "h_kv": hkv, "d_head": hd,
                           "mlp": inter, "vocab": vocab, "batch_per_gpu": B, "n": n, "d_s": 32, "n_codes": 4096,
                           "a": 16, "b": 4, "top_k": 256, "lm_head": "not run",
                           "parallelism": f"replicas x{world}"},
                "ssa_ms_per_step": attn_ms[0], "ssa_share": attn_ms[0] / ms_step, "output_finite": finite,
                "roofline": None, "cpu_baseline": None, "e2e": None, "clocks": clk}
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_decode(args):
    """Per-token decode time (``ssa_b200.decode.DecodeCache.step``: the new
    key's codes, one index append, routing of the query against the cache's
    index, sparse attention) at cache lengths 4k / 32k / 128k, config-3 heads
    (32 / 8 of 128, d_s 32, N_c 4096, a 16, b 4, k 256), batch 1, bf16.
    Beside it, the same step with the index rebuilt from every cached key
    (``route_with_key_codes``), which is what a decode loop without an
    incremental index does.  CUDA events around ``--steps`` consecutive steps."""
    import torch

    import ssa_b200 as ssa
    from ssa_b200 import _lib as L
    from ssa_b200 import workloads as W
    from ssa_b200.decode import DecodeCache

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    steps = max(args.steps, 10)
    res = {}
    for n in (4096, 32768, 131072):
        shape = W.Shape(**{**W.CONFIG3.asdict(), "n": n + steps})
        t = W.make_inputs(shape, seed=args.seed, dtype=torch.bfloat16, device=dev, planted=False,
                          generate_on_device=True)
        r = ssa.CodebookRouter(head_dim=shape.d, route_dim=shape.d_s, num_kv_heads=shape.h_kv,
                               num_codebook=shape.n_codes, codes_per_key=shape.b, codes_per_query=shape.a,
                               top_k=shape.top_k).to(dev)
        with torch.no_grad():
            r.W_qr.weight.copy_(t["w_qr"])
            r.W_kr.weight.copy_(t["w_kr"])
            r.codebook.copy_(t["codebook"])
        q, k, v = t["q"], t["k"], t["v"]
        cache = DecodeCache(r, 1, capacity=n + steps + args.warmup, num_q_heads=shape.h_q, device=dev)
        cache.append(k[:, :n - args.warmup], v[:, :n - args.warmup])
        p = n - args.warmup
        for _ in range(args.warmup):
            cache.step(q[:, p:p + 1], k[:, p:p + 1], v[:, p:p + 1])
            p += 1
        rebuilds0 = cache.rebuilds
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            cache.step(q[:, p:p + 1], k[:, p:p + 1], v[:, p:p + 1])
            p += 1
        e1.record()
        torch.cuda.synchronize(dev)
        ms_inc = e0.elapsed_time(e1) / steps
        rebuilds = cache.rebuilds - rebuilds0
        # the index upkeep alone: one append launch (device time) ...
        first = cache.n - 1
        args1 = cache._args(cache.n)
        st = torch.cuda.current_stream(dev).cuda_stream
        lib = L.lib()
        # re-appending the last key: the bucket ends are put back after each
        # timed call so the live index is not changed
        saved_end = cache.ix_end.clone()
        ms_append = _device_ms(lambda: L.check("append", lib.ssa_decode_index_append(
            ctypes.byref(args1), ctypes.byref(cache.index), first, 1, st)), dev, reps=1,
            after=lambda: cache.ix_end.copy_(saved_end))
        # ... against the full index build over every cached key
        codes_now = cache.codes[:, :cache.n].contiguous()
        ms_build = _device_ms(lambda: r.key_index(codes_now), dev)
        # the same decode steps with the index rebuilt from every cached key
        codes = cache.codes[:, :p]
        e0.record()
        for s in range(steps):
            pos = n + s
            r.key_codes(k[:, pos:pos + 1])                 # the new key's codes, as the incremental step does
            idx = r.route_with_key_codes(q[:, pos:pos + 1], k[:, :pos + 1], codes[:, :pos + 1], causal=True,
                                         q_offset=pos, index_dtype=torch.int32)
            ssa.sparse_exact_attention(q[:, pos:pos + 1], k[:, :pos + 1], v[:, :pos + 1], idx, is_causal=True,
                                       q_offset=pos)
        e1.record()
        torch.cuda.synchronize(dev)
        ssa.check_errors(dev)
        res[str(n)] = {"ms_per_token": ms_inc, "rebuilds_in_timed_steps": rebuilds,
                       "index_append_ms": ms_append, "full_index_build_ms": ms_build,
                       "ms_per_token_rebuilding_the_index": e0.elapsed_time(e1) / steps}
        del cache, t, q, k, v
        torch.cuda.empty_cache()
    print(json.dumps({"metric": "SSA decode ms per token (batch 1, config-3 heads, bf16)", "unit": "ms",
                      "higher_is_better": False, "steps": steps, "warmup": args.warmup,
                      "per_cache_length": res,
                      "note": "ms_per_token: DecodeCache.step (key codes, index append, routing, attention); "
                              "index_append_ms / full_index_build_ms: device time of the index upkeep per token "
                              "against a build over every cached key; ms_per_token_rebuilding_the_index: the same "
                              "steps through route_with_key_codes, which builds the index of all cached keys"}),
          flush=True)
    return 0


def _device_ms(fn, dev, reps=10, after=None):
    """Mean device time of ``fn`` (CUDA events around each call; ``after``
    runs between calls, outside the events)."""
    import torch

    tot = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize(dev)
        tot += e0.elapsed_time(e1)
        if after is not None:
            after()
    return tot / reps


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "decode":
        return run_decode(args)
    if args.workload == "config4":
        return run_config4(args)
    if args.workload == "config5":
        return run_config5(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
