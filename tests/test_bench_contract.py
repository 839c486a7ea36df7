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


def test_reference_arm_loads_no_product_library():
    """The CPU arm runs the reference's path only: after it has run, the
    process has mapped no shared object of fast_b200 (the product's C-ABI
    library and its drop-in modules); the reference sampler built from its own
    source (oracle/_ref) or the C restatement are the only native code."""
    code = "\n".join([
        "import runpy, sys",
        "sys.argv = %r" % (["bench.py"] + CMD[2:]),
        "try:",
        "    runpy.run_path('bench.py', run_name='__main__')",
        "except SystemExit:",
        "    pass",
        "libs = {ln.split()[-1] for ln in open('/proc/self/maps') if ln.rstrip().endswith('.so')}",
        "mods = sorted(m for m in sys.modules if m.startswith('fast_b200'))",
        "print('PRODUCT_SO' if any('/fast_b200/' in p for p in libs) else 'NO_PRODUCT_SO', mods)",
    ])
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=dict(os.environ, RANK="0"), capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "NO_PRODUCT_SO" in r.stdout, r.stdout[-2000:]
    assert "fast_b200.capi" not in r.stdout and "fast_b200.ops" not in r.stdout


def test_both_arms_describe_the_workload_alike():
    """The reference arm's `config` object is the one the fast arm prints for
    the same arguments (bench_config), so the two lines compare the same
    workload; arm-specific settings live outside it."""
    sys.path.insert(0, ROOT)
    import importlib
    bench = importlib.import_module("bench")
    from fast_b200.data import CONFIGS
    ns = type("A", (), dict(data=None, edges=None))()
    for c, world in ((5, 1), (5, 8), (2, 4)):
        cfg = CONFIGS[c]
        B, gB = bench.batch_sizes(cfg, world)
        d = bench.bench_config(ns, cfg, world, B, gB)
        assert d["global_batch"] == gB and d["local_batch"] * world == gB and d["parallelism"] == "dp%d" % world
        assert "l2" in d and not {"gemm", "launch", "step", "precision"} & set(d)


def test_oracle_parameter_tree_mirrors_the_product():
    """oracle/ref_model.py (the CPU arm's parameters) has the reference
    GeneralModel's module tree: the product model's state_dict loads into it
    strictly, for 1- and 2-layer TGAT with and without node features."""
    import torch
    from fast_b200.model import GeneralModel as Product
    from oracle.ref_model import GeneralModel as Ref
    for layers, dn, de in ((2, 0, 172), (1, 100, 100), (2, 413, 186)):
        sp = dict(layer=layers, neighbor=[10] * layers, strategy="recent", prop_time=False, history=1, duration=0)
        gp = dict(arch="transformer_attention", layer=layers, att_head=2, dim_time=100, dim_out=100)
        tp = dict(lr=1e-4, dropout=0.1, att_dropout=0.1)
        mp = dict(type="none", dim_out=0)
        a, b = Product(dn, de, sp, mp, dict(gp), tp), Ref(dn, de, sp, mp, dict(gp), tp)
        sa, sb = a.state_dict(), b.state_dict()
        assert sorted(sa) == sorted(sb)
        assert all(sa[k].shape == sb[k].shape for k in sa)
        b.load_state_dict(sa, strict=True)
        assert torch.equal(b.layers["l0h0"].time_enc.w.weight, a.layers["l0h0"].time_enc.w.weight)
