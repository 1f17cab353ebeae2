"""Full-chain forward+backward throughput (Mpixels/s) of the differentiable
rasterization chain on B200, one process per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg4] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

A step is one pass of the configuration's chain (rasterize -> interpolate ->
texture -> antialias -> MSE, then every VJP) over the rank's views, plus the
NCCL all-reduce of the shared-parameter gradients when N > 1.  Rank 0 prints
one JSON line.  The default workload is configuration 4 of the benchmark
(1M-triangle soup, 32 views at 1024^2, two depth-peeled layers with rast_db,
8-channel interpolation with diffAttrs=.all, antialias with the topology hash),
the configuration the throughput target is stated on.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mlx-swift-diffrast_b200"))
sys.path.insert(0, ROOT)

METRIC = "full-chain fwd+bwd Mpixels/s"

WORKLOADS = {
    "cfg1": "tier-1 colour fit: 1 triangle, N=1, 256^2, rasterize->interpolate(RGB)->antialias->MSE, bwd d_pos/d_rgb",
    "cfg2": "icosphere L4 (2562 v / 5120 t), 8 views 512^2, RGB+UV interpolate, bilinear clamp 512^2x3 texture, "
            "antialias, MSE; bwd d_pos/d_attr/d_tex",
    "cfg3": "icosphere L4, 16 views 1024^2, rast_db, UV diffAttrs=.all, trilinear 2048^2x4 wrap texture with per-pixel "
            "mip bias, MSE; bwd d_tex(all levels)/d_uv/d_uvDA->d_pos",
    "cfg4": "1M-triangle soup (20% in edge-sharing strips), 32 views/GPU at 1024^2, 2 depth-peeled layers with rast_db, "
            "interpolate A=8 diffAttrs=.all, antialias+topology hash, MSE; bwd d_pos(->shared verts)/d_attr",
    "cfg5": "geodesic sphere 499,280 tris, 256 views 2048^2 sharded over GPUs, rast_db, normals diffAttrs=.all, "
            "trilinear cube 6x1024^2x3 (an extension of the reference: face pyramids, LOD from the normals' "
            "derivatives), antialias, MSE; bwd d_verts/d_tex(all levels)",
}
CFG5_LINEAR = ("geodesic sphere 499,280 tris, 256 views 2048^2 sharded over GPUs, cube 6x1024^2x3 in the reference's "
               ".linear mode, antialias, MSE; bwd d_verts/d_tex")
def workload_text(args) -> str:
    if args.config == "cfg5" and args.cube_filter == "linear":
        return CFG5_LINEAR
    return WORKLOADS[args.config]


# Configurations whose per-GPU work is fixed as N grows (each rank renders the
# configuration's full view count); cfg5 splits its 256 views over the ranks.
WEAK = {"cfg1", "cfg2", "cfg3", "cfg4"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------- algorithmic bytes

# Measured DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of each
# library kernel in one full-size cfg4 step (32 views x 1024^2 = P4 pixels per
# layer), summed over the kernel's launches in the step, per pixel.  They come
# from NCU_CAPTURE: ncu collects these three metrics in one pass, so the
# capture replays nothing and sees the step's real cache state (tables that
# a kernel gathers from and that miss L2 once per view, such as the raster
# VJP's vertex rows, are understated by a smaller capture).  Scaled by the
# pixels of a run with other view counts.
P4 = 32 * 1024 * 1024
NCU_CAPTURE = {
    "commit": "66ceb2f",
    "command": ("ncu --metrics gpu__time_duration.sum,dram__bytes_read.sum,dram__bytes_write.sum "
                "--clock-control none -c 200 --csv python -u bench.py --steps 1 --warmup 3 --no-e2e --no-cpu"),
}
NCU_DRAM_BYTES_PER_PIXEL = {
    ("cfg4", "raster_setup"): 1901652736 / P4,
    ("cfg4", "raster_scatter"): 1344560640 / P4,
    ("cfg4", "raster_tiles_interp"): 14772549632 / P4,
    ("cfg4", "aa_fwd"): 4542650880 / P4,
    ("cfg4", "aa_fwd_edges"): 1170285312 / P4,
    ("cfg4", "aa_bwd"): 3962484480 / P4,
    ("cfg4", "aa_bwd_edges"): 964109056 / P4,
    ("cfg4", "interp_raster_bwd"): 5654321664 / P4,  # both layers, one launch
}


def algorithmic_bytes(cfg: str, chain) -> dict:
    """Compulsory HBM bytes per step for each library kernel (each input read
    once, each output written once; intermediates such as setup records, tile
    lists and scan buffers count zero).  Returns {kernel: bytes per step}."""
    import torch  # noqa: F401
    i = chain.info
    n = i.n_views
    H, W = i.res
    P = n * H * W
    k = {}

    def add(name, b):
        k[name] = k.get(name, 0) + b

    def add_aa(C, V, T, nv):
        """Antialias fused with its MSE: the forward reads colour, rast and the
        target and writes out plus the 17 B/px silhouette record; the VJP reads
        the record, out and the target (the loss's cotangent is formed from
        them) and writes d_color.  nv: vertex batches read (1 with per-view
        transforms of one shared buffer)."""
        add("aa_fwd", P * (12 * C + 16 + 17) + nv * V * 16 + 2 * T * 12)
        add("aa_bwd", P * (12 * C + 17) + 2 * nv * V * 16 + 2 * T * 12)

    if cfg == "cfg4":
        V, T, A = chain.base.shape[0], chain.tri.shape[0], 8
        # Vertices are the shared [V, 4] soup (Nv = 1) transformed per view in-kernel.
        add("raster_setup", V * 16 + T * 12)  # both layers share setup and tile lists
        # One tile pass writes both layers (rast + rast_db each); layer 0 is never re-read.
        fused = getattr(chain, "fused", False)
        from diffrast import ops
        fused_vjp = fused and ops.FUSED_LAYERS_VJP
        add("raster_tiles_interp" if fused else "raster_tiles", 2 * (P * 16 + P * 16))
        if fused_vjp:
            # One launch for both layers' VJPs: attr and verts read, d_attr and
            # d_verts written once; per layer its rast and out's cotangent.
            add("interp_raster_bwd", 2 * V * A * 4 + 2 * V * 16 + T * 12)
        for layer in (0, 1):
            # Layer 1's interpolation also reads its MSE target (the fused loss).
            # Fused into the tile pass, it reads no rast / rast_db back.
            if fused:
                add("raster_tiles_interp", V * A * 4 + T * 12 + P * (4 * A + 8 * A) + (P * 4 * A if layer else 0))
            else:
                add("interp_fwd", V * A * 4 + T * 12 + P * (16 + 16 + 4 * A + 8 * A) + (P * 4 * A if layer else 0))
            # out_da never reaches the loss: the VJP runs without the DA terms.
            # Layer 0 reads d_out; layer 1 forms it from its output and target.
            if fused_vjp:
                # rast once; d_rast stays in registers.
                add("interp_raster_bwd", P * (16 + 4 * A) + (P * 4 * A if layer else 0))
                continue
            add("interp_bwd", 2 * V * A * 4 + T * 12 + P * (16 + 16 + 4 * A) + (P * 4 * A if layer else 0))
            # rast_db's cotangent is zero (out_da is off the loss path): not read.
            add("raster_bwd", 2 * V * 16 + T * 12 + P * 32)
        add_aa(A, V, T, 1)
    elif cfg == "cfg1":
        V, T, C = 3, 1, 3
        add("raster_setup", V * 16 + T * 12)
        add("raster_tiles", P * 16)
        add("interp_fwd", V * C * 4 + T * 12 + P * (16 + 4 * C))
        add("interp_bwd", 2 * V * C * 4 + T * 12 + P * (32 + 4 * C))
        add("raster_bwd", 2 * V * 16 + T * 12 + P * 32)
        add_aa(C, V, T, 1)
    elif cfg == "cfg2":
        V, T = chain.pos.shape[1], chain.tri.shape[0]
        S = 512 * 512 * 3 * 4
        add("raster_setup", n * V * 16 + T * 12)
        add("raster_tiles", P * 16)
        add("interp_fwd", V * 3 * 4 + V * 2 * 4 + 2 * T * 12 + P * (16 + 12) + P * (16 + 8))
        add("interp_bwd", 2 * V * 5 * 4 + 2 * T * 12 + P * (32 + 12) + P * (32 + 8))
        add("tex_linear_fwd", S + P * (8 + 12))
        add("tex_linear_bwd", 2 * S + P * (16 + 12))
        add("raster_bwd", 2 * n * V * 16 + T * 12 + P * 32)
        add_aa(3, V, T, n)
    elif cfg == "cfg3":
        V, T = chain.pos.shape[1], chain.tri.shape[0]
        S0 = 2048 * 2048 * 4 * 4
        S_all = S0 * 4 // 3
        add("raster_setup", n * V * 16 + T * 12)
        add("raster_tiles", P * 32)
        add("interp_fwd", V * 2 * 4 + T * 12 + P * (16 + 16 + 8 + 16))
        add("interp_bwd", 2 * V * 2 * 4 + T * 12 + P * (32 + 32 + 8 + 16))
        add("mip_down", S0 + S0 // 3)
        add("tex_mip_fwd", S_all + P * (8 + 16 + 4 + 16))
        add("tex_mip_bwd", 2 * S_all + P * (16 + 32 + 4 + 16))
        add("mip_fold", S_all + S0)
        add("raster_bwd", 2 * n * V * 16 + T * 12 + P * 32 + P * 16)
        add("mse", P * 8 * 4)  # loss: read pred and target
        add("mse_bwd", P * 12 * 4)  # read pred and target, write d_pred
    elif cfg == "cfg5":
        V, T = chain.verts.shape[0], chain.tri.shape[0]
        S = 6 * 1024 * 1024 * 3 * 4
        micro = -(-n // chain.micro)
        add("raster_setup", n * V * 16 + micro * T * 12)
        if chain.filter_mode == 1:  # the reference's .linear cube
            add("raster_tiles", P * 16)
            add("interp_fwd", micro * (V * 12 + T * 12) + P * (16 + 12))
            add("interp_bwd", micro * (2 * V * 12 + T * 12) + P * (32 + 12))
            add("tex_cube_fwd", micro * S + P * (12 + 12))
            add("tex_cube_bwd", micro * 2 * S + P * (12 + 12 + 12))
            add("raster_bwd", 2 * n * V * 16 + micro * T * 12 + P * 32)
        else:  # trilinear: rast_db, dirDA (6 floats / px), the faces' pyramids
            S_all = S * 4 // 3
            add("raster_tiles", P * 32)
            add("interp_fwd", micro * (V * 12 + T * 12) + P * (32 + 12 + 24))
            add("interp_bwd", micro * (2 * V * 12 + T * 12) + P * (32 + 12 + 24 + 32))
            add("mip_down", micro * (S + S // 3))
            add("tex_cube_mip_fwd", micro * S_all + P * (12 + 24 + 12))
            add("tex_cube_mip_bwd", micro * 2 * S_all + P * (12 + 24 + 12 + 12 + 24))
            add("mip_fold", micro * (S_all + S))
            add("raster_bwd", 2 * n * V * 16 + micro * T * 12 + P * (32 + 16))
        add_aa(3, V, micro * T, micro)  # per-view transforms of the shared vertices
    return k


# --------------------------------------------------------- CPU baseline

def cpu_chain_sample(cfg: str, nthreads: int, cube_filter: str = "trilinear"):
    """Build a bounded sample of the configuration for the CPU oracle chain.
    Returns (callable, pixels, description)."""
    import numpy as np

    import oracle
    import oracle.chains as OC
    from diffrast import scenes

    if cfg == "cfg4":
        s = scenes.scene_cfg4(n_views=1)
        pos = np.einsum("nij,vj->nvi", s["sim"], s["base"]).astype(np.float32)
        g = np.random.default_rng(13)
        H, W = s["res"]
        t0 = g.normal(size=(1, H, W, 8)).astype(np.float32)
        t1 = g.normal(size=(1, H, W, 8)).astype(np.float32)
        topo = oracle.topology_hash(s["tri"])
        f = lambda: OC.cfg4(pos, s["tri"], s["attr"], t0, t1, s["res"], topo, nthreads)  # noqa: E731
        return f, H * W, "1 of 32 views of cfg4 at full size (1M triangles, 1024^2, 2 layers, A=8, aa)"
    if cfg == "cfg1":
        s = scenes.scene_cfg1()
        topo = oracle.topology_hash(s["tri"])
        f = lambda: OC.cfg1(s["pos"], s["tri"], s["attr"], s["target"], s["res"], topo, nthreads)  # noqa: E731
        return f, 256 * 256, "full cfg1 step"
    if cfg == "cfg2":
        s = scenes.scene_cfg2()
        topo = oracle.topology_hash(s["tri"])
        f = lambda: OC.cfg2(s["pos"][:2], s["tri"], s["rgb"], s["uv"], s["tex"], s["target"][:2], s["res"], topo,  # noqa: E731
                            nthreads)
        return f, 2 * 512 * 512, "2 of 8 views of cfg2"
    if cfg == "cfg3":
        s = scenes.scene_cfg3()
        f = lambda: OC.cfg3(s["pos"][:1], s["tri"], s["uv"], s["tex"], s["bias_map"][:1], s["target"][:1],  # noqa: E731
                            s["res"], nthreads)
        return f, 1024 * 1024, "1 of 16 views of cfg3"
    s = scenes.scene_cfg5(n_views=1)
    pos = scenes.clip_positions(s["verts"], s["mvps"][:1])
    g = np.random.default_rng(16)
    tgt = g.random((1,) + s["res"] + (3,)).astype(np.float32)
    topo = oracle.topology_hash(s["tri"])
    fm = "linear" if cube_filter == "linear" else "linear-mipmap-linear"
    f = lambda: OC.cfg5(pos, s["tri"], s["unit"], s["cube"], tgt, s["res"], topo, nthreads, fm)  # noqa: E731
    return f, s["res"][0] * s["res"][1], f"1 of 256 views of cfg5 ({cube_filter} cube)"


def time_cpu(cfg: str, reps: int = 2, cube_filter: str = "trilinear"):
    nthreads = os.cpu_count() or 1
    f, pixels, desc = cpu_chain_sample(cfg, nthreads, cube_filter)
    f()  # warm-up (oracle scratch pool, page faults)
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        f()
        ts.append(time.perf_counter() - t0)
    dt = statistics.median(ts)
    return {"value": pixels / dt / 1e6, "unit": "Mpx/s", "cores": nthreads, "kind": "port",
            "sample": f"{desc}; median of {reps} runs after 1 warm-up, {dt:.2f} s each"}


# ------------------------------------------------------------------ main

def dist_setup(args):
    from diffrast import dist as D
    return D.init_from_env(timeout_s=300.0)


def run_reference(args, ws, rank):
    """The reference's path on the host: the oracle's restatement of the
    reference kernels (the reference itself is Swift + Metal and cannot run on
    this machine), with every host thread, each step a bounded sample."""
    if rank != 0:
        return
    nthreads = os.cpu_count() or 1
    f, pixels, desc = cpu_chain_sample(args.config, nthreads, args.cube_filter)
    for _ in range(args.warmup):
        f()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        f()
    dt = (time.perf_counter() - t0) / args.steps
    v = pixels / dt / 1e6
    line = {"metric": METRIC, "value": v, "unit": "Mpx/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak" if args.config in WEAK else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded PCG64 scenes)", "impl": "reference",
            "config": {"workload": f"{args.config}: {workload_text(args)}", "sample_per_step": desc},
            "cpu_baseline": {"value": v, "unit": "Mpx/s", "cores": nthreads, "kind": "port",
                             "sample": desc + " per step; CPU oracle restatement of the reference kernels"},
            "e2e": {"value": v, "unit": "Mpx/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="cfg4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--views", type=int, default=0, help="override views per GPU (profiling runs)")
    ap.add_argument("--graph", action="store_true",
                    help="single GPU: capture one step in a CUDA graph (fixed tile-list capacity, no host readback) "
                         "and time its replays; the per-kernel breakdown comes from an eager pass")
    ap.add_argument("--list-capacity", type=int, default=1 << 26,
                    help="tile-list capacity in (tile, triangle) pairs for --graph")
    ap.add_argument("--cube-filter", default="trilinear", choices=["trilinear", "linear"],
                    help="cfg5: trilinear cube (the configuration's text; an extension of the reference) or the "
                         "reference's own .linear cube mode")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl == "ours" else args.warmup

    ws, rank, local = dist_setup(args)
    if args.impl == "reference":
        run_reference(args, ws, rank)
        if ws > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch
    import torch.distributed as dist

    import diffrast
    from diffrast import _lib, chains

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    cfg = args.config
    from diffrast import dist as D
    total = args.views or chains.TOTAL_VIEWS[cfg]
    lo, hi, tot = D.view_range(total, rank, ws, weak=cfg in WEAK)
    kw = {}
    if cfg == "cfg4":
        kw = dict(view_lo=lo, view_hi=hi, total_views=tot)
    elif cfg != "cfg1":
        kw = dict(view_lo=lo, view_hi=hi)
    if cfg == "cfg5" and args.cube_filter == "linear":
        kw["filter_mode"] = diffrast.FilterMode.linear
    chain = chains.CHAINS[cfg](dev, **kw)
    torch.cuda.synchronize()

    # Shared-parameter gradients are summed across ranks by all-reduces that
    # the backward launches as each gradient becomes final (overlapping the
    # rest of the backward); the step waits for them at its end.
    sync = D.GradSync(chain.shared_params())
    chain.grad_sync = sync

    # With several ranks, the time the stream waits at the end of a step for
    # the gradient all-reduces still in flight (CUDA events around the wait,
    # recorded during the timed steps).
    exposed = {"on": False, "events": []}

    def allreduce():
        if exposed["on"]:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            sync.finish()
            b.record()
            exposed["events"].append((a, b))
        else:
            sync.finish()

    def one_step():
        chain.zero_grad()
        loss = chain.step()
        allreduce()
        return loss

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    diffrast.sync(local)
    if ws > 1:
        dist.barrier()

    graph = None
    if args.graph:
        if ws > 1:
            raise SystemExit("--graph is single-GPU only")
        # Fixed list capacity: rasterize reads nothing back, so the whole step
        # (forward, every VJP) can be captured.  Warm up on a side stream (all
        # workspaces reach their size), then capture one step.
        diffrast.set_raster_list_capacity(args.list_capacity, local)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(3):
                one_step()
        torch.cuda.current_stream(dev).wait_stream(side)
        chain.zero_grad()
        graph = torch.cuda.CUDAGraph()
        n0 = diffrast.launch_count(local)
        with torch.cuda.graph(graph):
            static_loss = one_step()
        graph_launches = diffrast.launch_count(local) - n0
        for _ in range(args.warmup):
            graph.replay()
        torch.cuda.synchronize()

    def timed(step, timing):
        """CUDA-event time per step over args.steps steps (barriers and
        synchronisation on both sides), launches, per-kernel report."""
        if timing:
            _lib.set_timing(True, local)
        launches0 = diffrast.launch_count(local)
        stream = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            out = step()
        e1.record(stream)
        torch.cuda.synchronize()
        rep = None
        if timing:
            rep = _lib.timing_report(local)
            _lib.set_timing(False, local)
        return e0.elapsed_time(e1) / args.steps, diffrast.launch_count(local) - launches0, rep, out

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.4)
    if graph is not None:
        def replay():
            graph.replay()
            return static_loss
        ms, _, _, loss = timed(replay, False)
        launches = graph_launches * args.steps
        ms_eager, _, report, _ = timed(one_step, True)
    else:
        exposed["on"] = ws > 1
        ms, launches, report, loss = timed(one_step, True)
        exposed["on"] = False
    clk = clocks.stop()
    exposed_ms = None
    if exposed["events"]:
        exposed_ms = D.max_over_ranks(sum(a.elapsed_time(b) for a, b in exposed["events"]) / len(exposed["events"]),
                                      device=dev)
    ms_max = D.max_over_ranks(ms, device=dev)
    diffrast.sync(local)
    overflow_tiles = diffrast.raster_overflow(local) if graph is not None else None

    pixels_all = chain.info.pixels * ws
    value = pixels_all / (ms_max * 1e-3) / 1e6

    peak, peak_kind = load_peaks()
    algo = algorithmic_bytes(cfg, chain)
    kernels = {}
    for name, (cnt, tot_ms) in sorted(report.items(), key=lambda kv: -kv[1][1]):
        b = algo.get(name, 0) * args.steps
        ach = b / (tot_ms * 1e-3) / 1e9 if (b and tot_ms > 0) else None
        per_px = NCU_DRAM_BYTES_PER_PIXEL.get((cfg, name))
        # Measured bytes over the same CUDA-event time: the rate the kernel
        # really drives HBM at (>= the algorithmic rate when it re-reads).
        nb = per_px * chain.info.pixels * args.steps if per_px else None
        ncu_gbs = nb / (tot_ms * 1e-3) / 1e9 if (nb and tot_ms > 0) else None
        kernels[name] = {"launches": cnt, "ms_per_launch": tot_ms / cnt,
                         "share": tot_ms / ((ms_eager if graph is not None else ms) * args.steps),
                         "algo_bytes_per_launch": (b / cnt) if b else 0,
                         "gbs": ach, "frac": (ach / peak) if ach else None,
                         "ncu_dram_bytes_per_launch": (nb / cnt) if nb else None,
                         "ncu_gbs": ncu_gbs, "ncu_frac": (ncu_gbs / peak) if ncu_gbs else None}
    dom = next((n for n in kernels if kernels[n]["gbs"]), None)
    roof = None
    if dom:
        kd = kernels[dom]
        roof = {"kernel": dom, "bound": "hbm", "achieved": kd["gbs"], "peak": peak, "unit": "GB/s",
                "frac": kd["frac"], "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": kd["ncu_dram_bytes_per_launch"],
                "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of this kernel in a full-size "
                                   f"cfg4 step, build {NCU_CAPTURE['commit']}, per pixel times this launch's pixels "
                                   f"({NCU_CAPTURE['command']})") if kd["ncu_dram_bytes_per_launch"] else None,
                "traffic_gbs": kd["ncu_gbs"], "traffic_frac": kd["ncu_frac"],
                "algo_bytes_per_launch": kd["algo_bytes_per_launch"]}

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(chain, cfg, args, ws, dev, allreduce)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        try:
            cpu = time_cpu(cfg, cube_filter=args.cube_filter)
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:200]}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "Mpx/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
                "scaling": "weak" if cfg in WEAK else "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded PCG64 scenes, seeded torch targets)",
                "config": {"workload": f"{cfg}: {workload_text(args)}", "views_per_gpu": chain.info.n_views,
                           "resolution": list(chain.info.res), "pixels_per_step": pixels_all,
                           "parallelism": f"dp{ws} (views sharded, grads all-reduced)" if ws > 1 else "single GPU",
                           "l2": ("inputs larger than L2 (per-step tensors are GBs; no flush needed)"
                                  if chain.info.pixels * 64 > 126e6 else
                                  "working set smaller than L2 and not flushed (a small configuration)")},
                "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
                "gpu_launches_per_step": launches / args.steps, "clocks": clk, "kernels": kernels,
                "allreduce_exposed_ms": exposed_ms,
                "loss": float(loss.detach())}
        if graph is not None:
            line["execution"] = {"cuda_graph": True, "list_capacity": args.list_capacity,
                                 "overflow_tiles": overflow_tiles, "eager_ms_per_step": ms_eager}
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(chain, cfg, args, ws, dev, allreduce):
    """Same step through the public API with host inputs: every step copies its
    per-view inputs (targets and view transforms) from pinned host memory and
    reads the loss back, inside the timed region.  As a training loop's loader
    would, the inputs of step k+1 are copied on a second stream into the other
    of two device buffer sets while step k computes; the last step's loss
    read-back closes the timed region."""
    import torch

    names = [n for n in chain_input_names(cfg) if getattr(chain, n, None) is not None]
    host = [getattr(chain, n).detach().cpu().pin_memory() for n in names]
    h2d = sum(t.numel() * t.element_size() for t in host)
    out = torch.empty((), dtype=torch.float32).pin_memory()
    stream = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(dev)
    bufs = [[getattr(chain, n) for n in names], [torch.empty_like(getattr(chain, n)) for n in names]]
    ready = [torch.cuda.Event(), torch.cuda.Event()]
    free = [torch.cuda.Event(), torch.cuda.Event()]

    def issue(slot):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[slot])  # the step that last read this set is done
            for d, h in zip(bufs[slot], host):
                d.copy_(h, non_blocking=True)
            ready[slot].record(copy_stream)

    def run(k):
        slot = k % 2
        stream.wait_event(ready[slot])
        for n, d in zip(names, bufs[slot]):
            setattr(chain, n, d)
        chain.zero_grad()
        loss = chain.step()
        allreduce()
        out.copy_(loss.detach(), non_blocking=True)
        free[slot].record(stream)

    def steps(k_total):
        copy_stream.wait_stream(stream)
        issue(0)
        for k in range(k_total):
            if k + 1 < k_total:
                issue((k + 1) % 2)
            run(k)

    steps(2)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    steps(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    for n, d in zip(names, bufs[0]):
        setattr(chain, n, d)
    from diffrast import dist as D
    ms = D.max_over_ranks(e0.elapsed_time(e1) / args.steps, device=dev)
    return {"value": chain.info.pixels * ws / (ms * 1e-3) / 1e6, "unit": "Mpx/s", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
            "inputs": "per-step targets and view transforms from pinned host memory, copied one step ahead "
                      "on a second stream (double-buffered); loss read back every step"}


def chain_input_names(cfg):
    if cfg == "cfg4":
        return ["tgt0", "tgt1", "sim"]
    if cfg == "cfg5":
        return ["target", "mvp"]
    if cfg == "cfg3":
        return ["target", "bias"]
    return ["target"]


if __name__ == "__main__":
    main()
