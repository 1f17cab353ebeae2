"""bench.py's output contract, checked on the CPU through its reference arm
(the oracle's restatement of the reference kernels on the host cores): one
JSON line with the metric, the configuration and the CPU baseline; under
torchrun only rank 0 prints and every rank exits 0."""
import json
import os
import subprocess
import sys

from conftest import ROOT

BENCH = os.path.join(ROOT, "bench.py")
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _env():
    env = dict(os.environ)
    env["CUDA_VISIBLE_DEVICES"] = ""
    return env


def _json_lines(out: str):
    return [json.loads(ln) for ln in out.splitlines() if ln.startswith("{")]


def _check_line(d):
    assert KEYS <= set(d), KEYS - set(d)
    assert d["impl"] == "reference" and d["metric"] == "full-chain fwd+bwd Mpixels/s"
    assert d["unit"] == "Mpx/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"].startswith("cfg1:")
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "Mpx/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, BENCH, "--impl", "reference", "--config", "cfg1", "--steps", "1",
                        "--warmup", "0"], capture_output=True, text=True, timeout=300, env=_env(), cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_line(lines[0])


def test_reference_arm_under_torchrun_prints_once():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29561", BENCH, "--impl", "reference",
           "--config", "cfg1", "--gpus", "2", "--steps", "1", "--warmup", "0"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=_env(), cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    _check_line(lines[0])
    assert lines[0]["n_gpus"] == 2


def test_bench_options():
    r = subprocess.run([sys.executable, BENCH, "--help"], capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert r.returncode == 0
    for opt in ("--gpus", "--steps", "--warmup", "--config", "--impl", "--graph", "--cube-filter"):
        assert opt in r.stdout
