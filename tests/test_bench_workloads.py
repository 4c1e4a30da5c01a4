"""Host-side pieces of bench.py's workloads (CPU).

The config-3 trace must be the reference's: generate_poisson_traffic
(benchmarks/traffic.py:23-55) called with 32 requests, 8 req/s, prompts
256-2048, 128 new tokens, seed 42 gives the prompt lengths and last arrival
pinned below (values produced by running the reference's function with those
arguments).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_poisson_trace_matches_reference_draws():
    t = bench.poisson_trace(32, 8.0, (256, 2048), (128, 128), 42)
    assert len(t) == 32
    assert [p for _, p, _ in t][:8] == [307, 541, 1372, 321, 732, 1722, 1462, 269]
    assert sum(p for _, p, _ in t) == 37034
    assert all(n == 128 for _, _, n in t)
    assert abs(t[-1][0] - 4.11) < 0.005
    arrivals = [a for a, _, _ in t]
    assert arrivals == sorted(arrivals)


def test_workload_table_names_the_baseline_configs():
    wl = bench.WORKLOADS
    assert wl["qwen05b-int8"]["prompt"] == 512 and wl["qwen05b-int8"]["new"] == 50
    cb = wl["qwen05b-int4-cb"]
    assert (cb["requests"], cb["rate"], cb["prompt_range"], cb["new"]) == (32, 8.0, (256, 2048), 128)
    assert wl["llama8b-int4"]["batch"] == 64 and wl["llama8b-int4"]["context"] == 4096
