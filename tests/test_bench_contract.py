"""bench.py's JSON contract on the host: the reference arm (the reference library's own CPU
FlatIndex::search_batch from oracle/_ref) prints one line with the keys the driver reads, on a
reduced workload so that it runs in seconds."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT


def test_reference_arm_line_has_the_contract_keys():
    from oracle.oracle import REF_SO
    if not os.path.exists(REF_SO):
        pytest.skip("oracle/_ref not built")
    import time
    t0 = time.perf_counter()
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--rows", "20000", "--queries", "300", "--steps", "2", "--warmup", "1"],
                         cwd=ROOT, capture_output=True, text=True, timeout=300)
    wall = time.perf_counter() - t0
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "data", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "QPS" and line["value"] > 0
    assert line["steps"] == 2 and line["warmup"] == 1 and line["higher_is_better"] is True
    assert line["config"]["global_batch"] == 300
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "QPS", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    # The line claims only the work it timed: ms_per_step is the measured time of a step that
    # searched queries_per_step queries, so the timed region fits in the run's wall time.
    per_step = line["queries_per_step"]
    assert 1 <= per_step <= 300
    assert abs(line["value"] - per_step / (line["ms_per_step"] / 1000.0)) <= 1e-6 * line["value"]
    assert line["ms_per_step"] * line["steps"] / 1000.0 < wall
    # The same workload description as the GPU arm prints for these arguments.
    sys.path.insert(0, ROOT)
    import argparse
    import bench
    args = argparse.Namespace(rows=20000, queries=300, workload="c1")
    assert line["config"] == bench.flat_config(args)


def test_bench_help_runs_without_a_gpu():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], cwd=ROOT,
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and "--shard" in out.stdout and "--workload" in out.stdout
