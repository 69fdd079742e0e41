"""The reference arm of bench.py on the CPU: `bench.py --impl reference` times the reference engine built from its own
sources (oracle/_ref) on the host cores and prints one JSON line with the GPU arm's metric, unit and config; under a
multi-rank launch only rank 0 runs and prints."""
import json
import os
import subprocess
import sys

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.skipif(not oracle.ref_available(), reason="the reference engine is not built")


def run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True, env=env,
                       cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_line():
    sys.path.insert(0, ROOT)
    import bench
    lines = run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "layer-tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == bench.WORKLOADS["decode"]["desc"]
    assert d["config"] == bench.layers_config(dict(bench.WORKLOADS["decode"]), 1)   # the GPU arm's config, key for key


def test_reference_arm_other_ranks_are_silent():
    assert run(["--impl", "reference", "--steps", "1", "--warmup", "0", "--gpus", "2"], {"RANK": "1", "WORLD_SIZE": "2"}) == []
