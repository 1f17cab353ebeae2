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


def _launched_names():
    import glob
    import re
    names = set()
    csrc = os.path.join(ROOT, "mlx-swift-diffrast_b200", "csrc")
    for f in glob.glob(os.path.join(csrc, "*.cu")) + glob.glob(os.path.join(csrc, "*.cuh")):
        names |= set(re.findall(r'DR_LAUNCHED\(ctx, "([a-z_0-9]+)"\)', open(f).read()))
    return names


def test_algorithmic_bytes_name_launched_kernels():
    # The roofline of every bench line divides these bytes by the CUDA-event
    # time of the kernel of the same name: every key must be a launched
    # kernel's name, every value positive, and each configuration's main
    # kernels present.
    from types import SimpleNamespace as NS

    import numpy as np

    import bench
    launched = _launched_names()

    def info(n, h, w):
        return NS(n_views=n, res=(h, w), pixels=n * h * w)

    z = np.zeros
    chains = {
        "cfg1": NS(info=info(1, 256, 256)),
        "cfg2": NS(info=info(8, 512, 512), pos=z((8, 2562, 4)), tri=z((5120, 3))),
        "cfg3": NS(info=info(16, 1024, 1024), pos=z((16, 2562, 4)), tri=z((5120, 3))),
        "cfg4": NS(info=info(32, 1024, 1024), base=z((2600000, 4)), tri=z((1000000, 3)), fused=True),
        "cfg4-separate": NS(info=info(32, 1024, 1024), base=z((2600000, 4)), tri=z((1000000, 3)), fused=False),
        "cfg5": NS(info=info(256, 2048, 2048), verts=z((249642, 4)), tri=z((499280, 3)), micro=16, filter_mode=3),
        "cfg5-linear": NS(info=info(256, 2048, 2048), verts=z((249642, 4)), tri=z((499280, 3)), micro=16,
                          filter_mode=1),
    }
    # The chains that end in antialias compute their MSE inside the antialias
    # kernels (and cfg4's layer-1 one inside interpolate): no mse launches.
    main = {"cfg1": {"raster_tiles", "interp_fwd", "interp_bwd", "raster_bwd", "aa_fwd", "aa_bwd"},
            "cfg2": {"tex_linear_fwd", "tex_linear_bwd", "interp_bwd", "aa_bwd"},
            "cfg3": {"tex_mip_fwd", "tex_mip_bwd", "mip_down", "mip_fold", "interp_bwd"},
            "cfg4": {"raster_tiles_interp", "interp_raster_bwd", "aa_fwd", "aa_bwd"},
            "cfg4-separate": {"raster_tiles", "interp_fwd", "interp_bwd", "raster_bwd", "aa_fwd", "aa_bwd"},
            "cfg5": {"tex_cube_mip_fwd", "tex_cube_mip_bwd", "mip_down", "mip_fold", "aa_bwd"},
            "cfg5-linear": {"tex_cube_fwd", "tex_cube_bwd", "aa_bwd"}}
    for name, ch in chains.items():
        b = bench.algorithmic_bytes(name.split("-")[0], ch)
        assert set(b) <= launched, (name, set(b) - launched)
        assert all(v > 0 for v in b.values()), name
        assert main[name] <= set(b), (name, main[name] - set(b))
        if name != "cfg3":
            assert not {"mse", "mse_bwd"} & set(b), name
