"""CPU: bench.py's reference arm keeps the JSON-line contract.

`--impl reference` times the reference's CPU path (the sampler built from the
reference's source, or its C restatement, plus the fp32 model) on the fast
arm's workload and prints one line with impl, metric, value, unit,
cpu_baseline and an e2e object without host<->device bytes.  Under torchrun
only rank 0 works; the other ranks exit 0 without output.  Config 1 (2,000
nodes, 1.3 M edges, zero features) keeps the run to seconds."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CMD = [sys.executable, "bench.py", "--impl", "reference", "--config", "1", "--steps", "2", "--warmup", "3"]


def _run(extra_env):
    env = dict(os.environ, **extra_env)
    return subprocess.run(CMD, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _run({"RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for k in ("metric", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config"):
        assert k in d, k
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["config"]["workload"] == "tgat1_lastfm_like"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("reference", "port") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
