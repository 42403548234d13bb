"""bench.py's reference arm on the CPU: `bench.py --impl reference` times the reference's own CPU
core (oracle/_ref/libref_core_fast.so: core/cpu_ops.cpp built unmodified, + the restated glue) on a
bounded sample of the serving workload and prints one JSON line with the GPU arm's metric, unit and
direction; under torchrun only rank 0 prints.  CPU only (the arm needs no GPU)."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REPO, "oracle", "_ref", "libref_core_fast.so")),
                                reason="oracle/_ref not built")


def _bench(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3",
                           "--cpu-seconds", "1"], cwd=REPO, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    sys.path.insert(0, REPO)
    import bench

    r = _bench({})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "libref_core_fast.so" in cb["sample"]
    # the sample's KV lengths are spread over the workload's draw: same mean within 5 %
    assert abs(cb["sample_mean_kv"] / cb["workload_mean_kv"] - 1) < 0.05
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_only_rank_zero_prints():
    r = _bench({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
