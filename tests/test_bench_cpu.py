"""The benchmark's reference arm on CPU: its JSON line reports the work it
really did (the measured time of each sampled step, the rows and heads of the
sample) and carries the same ``config`` dict as the GPU arm's line."""

import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_reference_arm_line_is_consistent():
    import bench
    from ssa_b200 import workloads as W

    n, steps = 512, 2
    t0 = time.perf_counter()
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--n", str(n),
                          "--steps", str(steps), "--warmup", "1"], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    wall = time.perf_counter() - t0
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads([x for x in out.stdout.splitlines() if x.startswith("{")][-1])
    assert line["impl"] == "reference" and line["steps"] == steps
    # the steps it claims fit in the time the process ran
    assert line["steps"] * line["ms_per_step"] / 1e3 <= wall
    # the same config dict the GPU arm prints for this workload
    shape = W.Shape(**{**W.CONFIG3.asdict(), "n": n})
    assert line["config"] == json.loads(json.dumps(bench.bench_config(shape, 1)))
    work = line["work_per_step"]
    assert work["kv_heads"] == 1 and work["query_rows"] == n // 4 and work["keys_coded"] == n
    assert line["cpu_baseline"]["value"] == line["value"] and line["e2e"]["h2d_bytes_per_step"] == 0
