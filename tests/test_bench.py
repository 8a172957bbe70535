"""bench.py's host-side pieces on the CPU: the CPU baseline line, the traffic
record it reads, and the config block both arms print."""

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_cpu_baseline_times_torch_cpu_operators_on_every_core():
    """The timed CPU baseline is torch's CPU operators over the given
    problems (here small ones), with the thread count and CPU model stated."""
    from emmy_ptx import workloads
    from oracle import torch_cpu
    probs = [workloads.build("rmsnorm", rows=64), workloads.build("softmax", rows=16)]
    cb = bench.cpu_baseline(probs, steps=3, warmup=1)
    assert cb["engine"] == "torch-cpu" and cb["kind"] == "port"
    assert cb["cores"] == torch_cpu.threads() and cb["value"] > 0 and cb["cpu"]
    assert str(sum(p.algorithmic_bytes() for p in probs)) in cb["sample"]


def test_traffic_comes_from_the_full_size_capture_and_scales_with_rows():
    rec = json.loads((ROOT / "profiles" / "traffic.json").read_text())["k_softmax_fused"]
    full = bench._traffic("k_softmax_fused", rec["algorithmic_bytes"])
    assert full["traffic"] == rec["dram_bytes_per_launch"]
    assert (ROOT / full["traffic_source"]).exists()
    shard = bench._traffic("k_softmax_fused", rec["algorithmic_bytes"] // 8)
    assert shard["traffic"] == pytest.approx(rec["dram_bytes_per_launch"] / 8, abs=1)
    assert bench._traffic("k_no_such_kernel", 1) == {"traffic": None}


def test_config_block_is_the_same_for_both_arms():
    """Both arms print the same config for a given N (the driver compares
    them); N > 1 names the exchange inside the step."""
    one, eight = bench.config_block(1), bench.config_block(8)
    assert one["workload"] == eight["workload"] == bench.WORKLOAD
    assert one["rows_per_rank"] == 8192 and eight["rows_per_rank"] == 1024
    assert "exchange" not in one and "NVLink" in eight["exchange"]
