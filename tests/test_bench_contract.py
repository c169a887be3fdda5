"""CPU checks of bench.py's output contract: the reference arm (the oracle
port timed on the host cores) prints one JSON line with the keys and types
the driver reads, and too few warm-up steps are refused.  No GPU is needed."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def run_bench(*args):
    env = dict(os.environ, RANK="0", WORLD_SIZE="1")
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=600, env=env, cwd=ROOT)


def test_reference_arm_prints_one_json_line(oracle_lib):
    p = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key, kind in (("metric", str), ("value", float), ("unit", str), ("n_gpus", int), ("steps", int),
                      ("warmup", int), ("ms_per_step", float), ("higher_is_better", bool), ("scaling", str),
                      ("dtype", str), ("data", str), ("config", dict), ("impl", str), ("cpu_baseline", dict),
                      ("e2e", dict)):
        assert isinstance(line[key], kind), key
    assert line["impl"] == "reference" and line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 3
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"]


def test_too_few_warmup_steps_are_refused():
    p = run_bench("--steps", "1", "--warmup", "2")
    assert p.returncode != 0 and "warmup" in (p.stderr + p.stdout)
