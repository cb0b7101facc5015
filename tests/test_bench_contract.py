"""bench.py's reference arm, the line the driver divides by (CPU only).

Rank 0 prints exactly one JSON line with the contract's keys, its
cpu_baseline describing the same run and an e2e block with no host copies;
other ranks of a torchrun launch exit 0 without work or output.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REQUIRED = {"metric", "value", "unit", "impl", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
            "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _run(env_extra, timeout):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout)


def _json_lines(stdout):
    return [json.loads(line) for line in stdout.splitlines() if line.startswith("{")]


def test_reference_arm_prints_one_contract_line():
    res = _run({}, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = _json_lines(res.stdout)
    assert len(lines) == 1
    line = lines[0]
    assert REQUIRED <= set(line), REQUIRED - set(line)
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["config"]["workload"] and line["config"]["seq_len"] == 32760
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["value"] == line["value"] and base["cores"] >= 1 and base["sample"]
    assert line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    # Every step's wall time is measured: the steps fit inside the arm's own run.
    assert line["ms_per_step"] * line["steps"] / 1e3 <= line["run_s"]
    # Same config object as the b200 arm of the same N, so the two lines compare.
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert line["config"] == json.loads(json.dumps(bench.workload_config(1)))
    cfg0 = base["config0_gloo_w2"]
    assert cfg0["world"] == 2 and cfg0["providers"]["math"]["ms_per_layer"] > 0


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}, timeout=120)
    assert res.returncode == 0, res.stderr[-2000:]
    assert not _json_lines(res.stdout)
