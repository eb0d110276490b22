"""bench.py's JSON line, checked on the CPU through the reference arm
(`--impl reference`, the oracle on the host cores): the keys the benchmark
contract names, the reference arm's own keys, and a world size above one
where only rank 0 prints."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def run(*args, env=None):
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, capture_output=True,
                         text=True, timeout=600, env=dict(os.environ, **(env or {})))
    assert res.returncode == 0, res.stderr[-2000:]
    return [line for line in res.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    [line] = run("--impl", "reference", "--workload", "mlp", "--steps", "1", "--warmup", "0")
    d = json.loads(line)
    assert KEYS <= set(d)
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["unit"] == "rows/s"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["config"]["workload"]


def test_reference_arm_other_ranks_print_nothing():
    assert run("--impl", "reference", "--workload", "mlp", "--steps", "1", "--warmup", "0",
               env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
