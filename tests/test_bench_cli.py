"""bench.py on the CPU: the reference arm of each activation workload (the oracle's restatement of
the reference's CPU path, timed on the host cores) prints one JSON line with the contract's keys,
so `bench.py --impl reference` works wherever the driver launches it."""

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "impl",
        "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload", ["kat_group_vitb_bf16", "bspline_kan", "kan_mlp_b16"])
def test_reference_arm_prints_the_contract_line(workload):
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--workload", workload, "--steps", "1", "--warmup", "0",
                          "--cpu-seconds", "0.5", "--ref-seconds", "2"],
                         cwd=REPO, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["n_gpus"] == 1
    assert d["config"]["workload"] == workload
    if workload == "kat_group_vitb_bf16":
        assert d["config"]["shape"] == [128, 197, 3072] and "sample_rows" in d
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["cores"] >= 1 and cpu["kind"] == "port"
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["unit"] == d["unit"]
