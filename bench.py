#!/usr/bin/env python3
"""Benchmark of the fused SH -> TP -> scatter interaction layer at 5000 atoms.

One step = neighbour list (PBC cell list) -> target/source CSR -> fused layer
forward -> backward (grads w.r.t. node features, weights and, through the edge
vectors, positions).  Workload: N=5000 atoms uniform in a periodic cube of side
44.3 A, cutoff 5 A (~150k edges), C=64, fp32, seed 3 (torch.manual_seed(3);
pos = rand(N,3)*L, W = randn(34,C,C)/sqrt(C), x = randn(N,C,16), upstream
grad = randn(N,C,16)), synthetic data.  The step runs as two CUDA graphs with no
host read inside the step: the neighbour list (count and fill into edge
buffers sized once, with headroom, from the first count) with the CSR views,
and the layer forward, backward and position gradient; every replay
recomputes everything from the current inputs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

--impl reference times the reference's own formulation of the same step on the
host CPU cores (normalise -> SH -> gather -> weighted TP -> index_add, torch
fp32, all threads, forward + autograd backward; benchmarks/benchmark_e2e_mace.py:323-350)
over a bounded sample of the target atoms, and reports the same metric.

With --gpus N > 1 (torchrun, one rank per GPU) the workload is the sharded
1M-atom system: N=1,000,000 atoms in a periodic cube of side 259 A, rc 5 A (~30M
edges), C=64, split into N slabs along x; every step each rank exchanges ghost
positions and features with its two neighbours over NCCL, runs the neighbour
list over its owned atoms' rows and the fused layer forward + backward, returns
ghost gradients to their owners and all-reduces dW (strong scaling).  Positions
and weights come from torch.manual_seed(4) as in config 5; node features and the
upstream gradient of the owned atoms are drawn on each rank's GPU (seed 4+rank).
--config 5 runs the same sharded step on one GPU (the T1 of the scaling).
The timed region is bracketed by a barrier; the max over ranks is reported.
"""
import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "batmobile-evo_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "fused SH+TP+scatter Medges/s at N=5k,C=64,L=3; % of roofline; 1/2/4/8 GPU"
CFG = dict(n=5000, box=44.3, rc=5.0, c=64, seed=3)
CFG5 = dict(n=1_000_000, box=259.0, rc=5.0, c=64, seed=4)
WORKLOAD = "config4: N=5000 atoms, periodic cube L=44.3, rc=5.0 (~150k edges), C=64, L_max=3; " \
           "step = neighbour list + fused layer fwd + bwd (grads x, W, pos)"


def make_inputs(cfg):
    torch.manual_seed(cfg["seed"])
    n, c = cfg["n"], cfg["c"]
    pos = torch.rand(n, 3) * cfg["box"]
    W = torch.randn(34, c, c) / math.sqrt(c)
    x = torch.randn(n, c, 16)
    G = torch.randn(n, c, 16)
    return pos, x, W, G


# ----------------------------------------------------------------- clocks --

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, index):
        self.index = index
        self.lines = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def wait_first(self, timeout=3.0):
        """Block until nvidia-smi has produced its first sample (its start-up
        takes longer than a short timed region)."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.01)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [s.strip() for s in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# -------------------------------------------------------------- GPU step --

class Stages:
    NAMES = ["neighbor_list", "csr", "layer_fwd", "layer_bwd", "pos_grad"]

    def __init__(self):
        self.ms = {k: 0.0 for k in self.NAMES}
        self.pending = []

    def mark(self, name, fn):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        r = fn()
        e.record()
        self.pending.append((name, s, e))
        return r

    def collect(self):
        for name, s, e in self.pending:
            self.ms[name] += s.elapsed_time(e)
        self.pending = []


def gpu_step(bm, _bm, pos, x, W, G, cfg, stages=None, lib=None, x_ready=None):
    box = [cfg["box"]] * 3
    if lib is not None:      # profiling: a boundary event before every API call
        def run(name, fn):
            lib.bm_profile_mark()
            return fn()
    else:
        run = stages.mark if stages else (lambda name, fn: fn())
    ei, vec, rp = run("neighbor_list", lambda: _bm.neighbor_list(pos, box, cfg["rc"], return_row_ptr=True))
    graph = run("csr", lambda: bm.EdgeGraph(ei, cfg["n"], src_row_ptr=rp, symmetric=True))
    if x_ready is not None:  # node features copied in on a side stream while the neighbour list ran
        torch.cuda.current_stream().wait_event(x_ready)
    out, slots = run("layer_fwd", lambda: _bm.layer_forward(x, vec, W, graph.src, graph.row_ptr_dst,
                                                            graph.perm_dst))
    rps, ps = graph.src_csr
    gx, gv, gw = run("layer_bwd", lambda: _bm.layer_backward(x, vec, W, graph.src, graph.dst, graph.row_ptr_dst,
                                                             graph.perm_dst, rps, ps, slots, G))
    gpos = run("pos_grad", lambda: _bm.edge_grad_to_pos(gv, graph.row_ptr_dst, graph.perm_dst, rps, ps))
    return out, gx, gw, gpos, ei.shape[1]


class GraphedStep:
    """The 5000-atom step as two CUDA graphs with no host read between them.
    Set-up (once): the neighbour-list count and one host read of the edge
    count E, which sizes static edge buffers with headroom (capacity).  Graph
    A: the neighbour-list count and fill into the capacity buffers and the CSR
    views (it needs no node features, so end to end it runs while they are
    still being copied in); graph B: the layer forward, backward and the
    position gradient.  Every replay recomputes everything from the current
    contents of the static inputs (positions, node features, weights, upstream
    gradient); the kernels walk the CSR offsets the replay computed, so only the
    first E slots of the buffers are touched.  A list longer than the capacity
    sets the device error flag (the fill drops what does not fit); `check()`
    reads it and `edges()` reads E, both outside the timed region.

    With `host` (pinned host tensors out, gx, gw, gpos) a third graph is captured
    for the end-to-end step: the same kernels, with the results copied to the
    host on a copy stream as soon as each is final (the layer output during the
    backward, the feature gradient during the edge-gradient pass), instead of
    after the step.  The backward runs as two API calls for that (feature
    gradient first, then edge and weight gradients); the device-resident graph
    uses the same split."""

    def __init__(self, bm, _bm, lib, cfg, pos, x, W, G, headroom=0.125, host=None):
        self.bm, self._bm, self.lib, self.cfg = bm, _bm, lib, cfg
        self.pos, self.x, self.W, self.G = pos, x, W, G
        self.plan = _bm.NeighborListPlan(pos, [cfg["box"]] * 3, cfg["rc"])
        self.plan.count()
        self.E = self.plan.num_edges()
        cap = self.E + int(self.E * headroom) + 1024
        dev = pos.device
        self.ei = torch.empty(2, cap, dtype=torch.int64, device=dev)
        self.vec = torch.empty(cap, 3, dtype=torch.float32, device=dev)
        self.capacity = cap
        self.graph_a = self._capture(self._edges)
        self.graph = self._out
        self.launches = self._captured_launches
        self.host = None
        self.graph_b = self._capture(self._layer)
        self.launches += self._captured_launches
        self.outputs = self._out
        self.graph_e2e = None
        if host is not None:
            self.host = host
            self.copy = torch.cuda.Stream(device=dev)
            self.graph_e2e = self._capture(self._layer)
            self.outputs_e2e = self._out

    def _capture(self, fn):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):   # one eager run first (one-time set-up inside the library)
            out = fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        l0 = self.lib.bm_launch_count()
        with torch.cuda.graph(g):
            out = fn()
        self._captured_launches = self.lib.bm_launch_count() - l0
        self._out = out
        return g

    def _edges(self):
        self.plan.count()
        self.plan.fill(self.ei, self.vec)
        graph = self.bm.EdgeGraph(self.ei, self.cfg["n"], src_row_ptr=self.plan.row_ptr, symmetric=True)
        graph.src_csr  # builds the source-grouped view inside this graph
        return graph

    def _to_host(self, name, t):
        if self.host is None:
            return
        self.copy.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.copy):
            self.host[name].copy_(t, non_blocking=True)

    def _layer(self):
        _bm, graph = self._bm, self.graph
        out, slots = _bm.layer_forward(self.x, self.vec, self.W, graph.src, graph.row_ptr_dst, graph.perm_dst)
        self._to_host("out", out)
        rps, ps = graph.src_csr
        args = (self.x, self.vec, self.W, graph.src, graph.dst, graph.row_ptr_dst, graph.perm_dst, rps, ps,
                slots, self.G)
        gx, _, _ = _bm.layer_backward(*args, needs_x=True, needs_v=False, needs_w=False)
        self._to_host("gx", gx)
        _, gv, gw = _bm.layer_backward(*args, needs_x=False, needs_v=True, needs_w=True)
        gpos = _bm.edge_grad_to_pos(gv, graph.row_ptr_dst, graph.perm_dst, rps, ps)
        self._to_host("gw", gw)
        self._to_host("gpos", gpos)
        if self.host is not None:
            torch.cuda.current_stream().wait_stream(self.copy)
        return out, gx, gw, gpos

    def __call__(self, x_ready=None, e2e=False):
        self.graph_a.replay()
        if x_ready is not None:  # node features copied in on a side stream meanwhile
            torch.cuda.current_stream().wait_event(x_ready)
        if e2e:  # results land in the pinned host tensors given at construction
            self.graph_e2e.replay()
            out, gx, gw, gpos = self.outputs_e2e
        else:
            self.graph_b.replay()
            out, gx, gw, gpos = self.outputs
        return out, gx, gw, gpos, self.E

    def edges(self):
        """E of the last replay (a host read)."""
        return self.plan.num_edges()

    def check(self):
        """Raises if a replay's list did not fit the capacity (or a device wait timed out)."""
        torch.cuda.synchronize()
        rc = self.lib.bm_device_error_check()
        if rc != 0:
            raise RuntimeError("graphed step: %s (capacity %d edges)" % (self.lib.bm_last_error().decode(),
                                                                          self.capacity))
        if self.edges() != self.E:
            raise RuntimeError("graphed step: the edge count changed (%d -> %d); rebuild the step"
                               % (self.E, self.edges()))


def mace_step_timing(bm, dev, pos, steps, warmup):
    """MACE-style model (reference MACEConfig: C = 32, 2 interaction blocks) on
    the config-4 positions: one step = neighbour list + energy + forces by
    autograd, inputs resident.  Reported beside the headline layer metric."""
    torch.manual_seed(5)
    model = bm.MACE(bm.MACEConfig()).to(dev)
    z = torch.randint(0, 89, (pos.shape[0],), device=dev)
    cell = torch.eye(3) * CFG["box"]
    for _ in range(warmup):
        model.energy_and_forces(pos, cell, z)
    torch.cuda.synchronize()
    times = []
    for _ in range(steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        model.energy_and_forces(pos, cell, z)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    ms = sum(times) / len(times)
    edges = model.graph(pos, cell)[0].num_edges
    return {"ms_per_step": ms, "edges": edges, "layers": 2, "channels": 32,
            "medges_per_s_per_layer": 2 * edges / (ms * 1e-3) / 1e6,
            "what": "embedding + 2 x (fused layer + Linear) + energy head, energy and forces (autograd), "
                    "neighbour list included; config-4 positions"}


def probe_fp32_tflops(lib):
    import ctypes
    buf = torch.zeros(1, device="cuda")
    iters, blocks = 4096, 148 * 8
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        lib.bm_probe_fp32(ctypes.c_void_p(buf.data_ptr()), iters, blocks, st)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 0.0
    for _ in range(5):
        s.record()
        lib.bm_probe_fp32(ctypes.c_void_p(buf.data_ptr()), iters, blocks, st)
        e.record()
        e.synchronize()
        flop = 2.0 * 8 * iters * blocks * 256
        best = max(best, flop / (s.elapsed_time(e) * 1e-3) / 1e12)
    return best


def probe_mma_tf32_tflops(lib):
    """Warp-level tf32 MMA rate (mma.sync m16n8k8) of this device, measured now."""
    import ctypes
    buf = torch.zeros(1, device="cuda")
    iters, blocks = 2048, 148 * 4
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        lib.bm_probe_mma_tf32(ctypes.c_void_p(buf.data_ptr()), iters, blocks, st)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = 0.0
    for _ in range(5):
        s.record()
        lib.bm_probe_mma_tf32(ctypes.c_void_p(buf.data_ptr()), iters, blocks, st)
        e.record()
        e.synchronize()
        flop = 2.0 * 16 * 8 * 8 * 8 * iters * blocks * 8   # 8 warps x 8 MMAs of 16x8x8 per iteration
        best = max(best, flop / (s.elapsed_time(e) * 1e-3) / 1e12)
    return best


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def layer_work(E, n_targets, n_sources, c):
    """Work per launch (FLOP, bounding unit) of the layer's kernels: 256*C FMA
    per edge for the edge sums (outer products or dY), run as a 3xTF32 product
    on the warp-level tensor cores (three tf32 MMAs per fp32 product: the
    tensor work is 3 x 2 x 256*C*E), 611*C per atom for the CG contraction (SIMT),
    156*C*C per atom for each channel mix."""
    return {
        "layer_bwd(target)": (3 * 2.0 * 256 * c * E, "mma"),
        "layer_fwd(aggregate)": (3 * 2.0 * 256 * c * E, "mma"),
        "layer_bwd(source aggregate)": (3 * 2.0 * 256 * c * E, "mma"),
        "tc_gemm(mix->irreps)": (2.0 * 156 * c * c * (n_targets + n_sources) / 2.0, "tensor"),
        "tc_gemm(grad->slots)": (2.0 * 156 * c * c * n_targets, "tensor"),
        "tc_gemm(weight grad)": (2.0 * 156 * c * c * n_targets, "tensor"),
    }


def roofline_of(kernels, work, mma_peak, tf32_peak, peak_kind, peaks, traffic=None):
    """The dominant kernel's achieved FLOP/s against its unit's measured peak."""
    top = next((k for k in kernels if k["name"] in work), kernels[0])
    flop, bound = work.get(top["name"], (0.0, "mma"))
    achieved = flop / (top["ms_per_launch"] * 1e-3) / 1e12
    peak = mma_peak if bound == "mma" else tf32_peak
    out = {
        "bound": "tensor", "unit": "TFLOP/s", "achieved": achieved, "peak": peak, "frac": achieved / peak,
        "traffic": (traffic or {}).get(top["name"]),
        "kernel": top["name"], "ms_per_launch": top["ms_per_launch"],
        "work": "%.3f GFLOP of tf32 MMA per launch (3 x the fp32 algorithmic 2*256*C*E)" % (flop / 1e9)
                if bound == "mma" else "%.3f GFLOP per launch (algorithmic)" % (flop / 1e9),
        "peak_source": ("warp-level tf32 mma.sync probe (bm_probe_mma_tf32) measured in this run"
                        if bound == "mma" else
                        "dense tf32 = MEASURED_PEAKS.json (%s) bf16 %.0f TF/s / 2" % (peak_kind,
                                                                                  peaks.get("bf16_tflops", 0))),
    }
    if bound == "mma":
        out["frac_of_dense_tf32"] = achieved / tf32_peak
        out["dense_tf32_source"] = "MEASURED_PEAKS.json (%s) bf16 %.0f TF/s / 2" % (peak_kind,
                                                                                 peaks.get("bf16_tflops", 0))
    return out


def kernel_table(nprof):
    from batmobile._lib import profile_report
    return sorted(({"name": nm, "launches_per_step": cnt / nprof, "ms_per_step": ms / nprof,
                    "ms_per_launch": ms / cnt} for nm, cnt, ms in profile_report()),
                  key=lambda k: -k["ms_per_step"])


# ---------------------------------------------------------- CPU baseline --

def cpu_reference_step(x, v, W, ei, n, Gs, sample_atoms):
    """The reference formulation, fp32 on the host: edges whose target is among
    the first `sample_atoms` atoms; forward + autograd backward (x, W, v)."""
    from oracle import ref_ops
    mask = ei[1] < sample_atoms
    eis = ei[:, mask]
    vs = v[mask].clone().requires_grad_(True)
    xs = x.clone().requires_grad_(True)
    Ws = W.clone().requires_grad_(True)
    out = ref_ops.interaction_chunked(xs, vs, Ws, eis, n, chunk=16384)
    out.backward(Gs)
    return int(eis.shape[1])


def cpu_full_step(pos, x, W, G, cfg):
    """The whole step on the host: neighbour list (the C cell list of the
    reference's brute-force predicate, one thread) + the reference
    formulation's forward and autograd backward over every edge, fp32."""
    from oracle import ref_ops
    t0 = time.perf_counter()
    ei, v = ref_ops.nl_cells(pos, [cfg["box"]] * 3, cfg["rc"])
    t_nl = time.perf_counter() - t0
    vs = v.clone().requires_grad_(True)
    xs = x.clone().requires_grad_(True)
    Ws = W.clone().requires_grad_(True)
    out = ref_ops.interaction_chunked(xs, vs, Ws, ei, cfg["n"], chunk=16384)
    out.backward(G)
    return int(ei.shape[1]), t_nl, time.perf_counter() - t0


def cpu_baseline(x, v, W, ei, G, n, budget_s=15.0, pos=None, cfg=None):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    xc, vc, Wc, eic, Gc = x.cpu(), v.cpu(), W.cpu(), ei.cpu(), G.cpu()
    if pos is not None:
        cpu_reference_step(xc, vc, Wc, eic, n, Gc, 250)  # warm-up on a sample
        edges, t_nl, t = cpu_full_step(pos.cpu(), xc, Wc, Gc, cfg)
        return {"value": edges / t / 1e6, "unit": "Medges/s", "cores": threads, "kind": "port",
                "ms_per_step": t * 1e3, "neighbor_list_ms": t_nl * 1e3,
                "sample": "the full step, one run: neighbour list (oracle C cell list, 1 thread) + reference PyTorch "
                          "formulation (oracle/ref_ops.interaction_chunked, fp32) forward + autograd backward "
                          "w.r.t. x, W, edge vectors over all %d edges" % edges}
    sample = 250
    t0 = time.perf_counter()
    edges = cpu_reference_step(xc, vc, Wc, eic, n, Gc, sample)  # warm-up
    dt = time.perf_counter() - t0
    reps = max(1, min(5, int(budget_s / max(dt, 1e-3))))
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        edges = cpu_reference_step(xc, vc, Wc, eic, n, Gc, sample)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": edges / t / 1e6, "unit": "Medges/s", "cores": threads, "kind": "port",
            "sample": "reference PyTorch formulation (oracle/ref_ops.interaction_chunked, fp32, fwd + autograd "
                      "bwd w.r.t. x, W, edge vectors) on the %d edges whose target is among the first %d of "
                      "the config-4 atoms; median of %d" % (edges, sample, reps)}


# ------------------------------------------------------------------ main --

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            dist.init_process_group(backend="nccl", device_id=torch.device("cuda", local),
                                    timeout=datetime.timedelta(seconds=300))
        else:
            dist.init_process_group(backend="gloo", timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def max_over_ranks(val, world):
    if world == 1:
        return val
    import torch.distributed as dist
    t = torch.tensor([val], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def run_reference(args, world, rank):
    if rank != 0:
        return
    pos, x, W, G = make_inputs(CFG)
    from oracle import ref_ops
    ei, v = ref_ops.nl_cells(pos, [CFG["box"]] * 3, CFG["rc"])
    vals = []
    info = None
    for i in range(args.warmup + args.steps):
        info = cpu_baseline(x, v, W, ei, G, CFG["n"], budget_s=4.0)
        if i >= args.warmup:
            vals.append(info["value"])
    val = statistics.median(vals)
    info["value"] = val
    line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "Medges/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD + " (CPU: bounded sample of target atoms)", "edges": int(ei.shape[1])},
            "cpu_baseline": info,
            "e2e": {"value": val, "unit": "Medges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def flush_l2(buf):
    """Evicts the L2 (126 MB) before a timed region: writes the 256 MB buffer,
    then reads it back, so that the lines left in L2 are clean ones of the
    flush buffer.  A write alone leaves about 126 MB of dirty lines whose
    write-back the next timed kernel would pay for as DRAM traffic of its own."""
    buf.zero_()
    torch.sum(buf, 0, out=_flush_sink(buf))


_SINKS = {}


def _flush_sink(buf):
    k = buf.device
    if k not in _SINKS:
        _SINKS[k] = torch.empty((), dtype=torch.float32, device=k)
    return _SINKS[k]


def timed_ops(ops, steps, warmup, flush):
    """CUDA-event time (ms, mean over `steps`) of each (name, fn) in order, the L2
    flushed before every op so each one reads its inputs from HBM."""
    tot = {name: 0.0 for name, _ in ops}
    for it in range(warmup + steps):
        for name, fn in ops:
            flush_l2(flush)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            if it >= warmup:
                tot[name] += s.elapsed_time(e)
    return {k: v / steps for k, v in tot.items()}


def run_ops_config(args, config):
    """Secondary single-GPU workloads (not the headline line):
    config 2 = spherical_harmonics + tensor_product_simple forward and backward on
    1M edges (HBM-bound: algorithmic bytes per op against the measured copy
    bandwidth); config 3 = weighted tensor_product forward + backward, N=1000,
    C_in=32, C_out=64 (latency-bound at this size)."""
    from batmobile import _batmobile as _bm
    from batmobile._lib import lib
    dev = torch.device("cuda", 0)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    peaks, peak_kind = measured_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    l0 = lib.bm_launch_count()
    if config == 2:
        torch.manual_seed(1)
        E = 1_000_000
        v = torch.randn(E, 3)
        v = v / v.norm(dim=1, keepdim=True)
        a = torch.randn(E, 16)
        g = torch.randn(E, 16)
        v, a, g = v.to(dev), a.to(dev), g.to(dev)
        st = {}
        st["Y"] = _bm.spherical_harmonics(v, 3)
        st["gy"] = _bm.tensor_product_simple_backward(a, st["Y"], g)[1]
        ops = [("spherical_harmonics", lambda: st.__setitem__("Y", _bm.spherical_harmonics(v, 3))),
               ("tensor_product_simple", lambda: _bm.tensor_product_simple(a, st["Y"])),
               ("tensor_product_simple_backward",
                lambda: st.__setitem__("gy", _bm.tensor_product_simple_backward(a, st["Y"], g)[1])),
               ("spherical_harmonics_backward", lambda: _bm.spherical_harmonics_backward(v, st["gy"]))]
        nbytes = {"spherical_harmonics": 12 + 64, "tensor_product_simple": 3 * 64,
                  "tensor_product_simple_backward": 3 * 64 + 2 * 64, "spherical_harmonics_backward": 12 + 64 + 12}
        ms = timed_ops(ops, args.steps, args.warmup, flush)
        # the four ops as one step (back to back, one event pair; the L2 flushed before the step)
        step = [("step", lambda: [fn() for _, fn in ops])]
        total = timed_ops(step, args.steps, args.warmup, flush)["step"]
        per_op = [{"op": k, "ms": ms[k], "bytes": nbytes[k] * E, "GB/s": nbytes[k] * E / (ms[k] * 1e-3) / 1e9,
                   "frac_of_hbm": nbytes[k] * E / (ms[k] * 1e-3) / 1e9 / hbm,
                   "note": "timed alone (L2 flushed before the op; includes its launch)"} for k in ms]
        line = {"metric": "config2: spherical_harmonics + tensor_product_simple fwd/bwd, E=1e6, L_max=3",
                "value": E / (total * 1e-3) / 1e6, "unit": "Medges/s", "ms_per_step": total, "steps": args.steps,
                "warmup": args.warmup, "dtype": "f32", "data": "synthetic (seed 1)",
                "roofline": {"bound": "hbm", "unit": "GB/s", "achieved": 676 * E / (total * 1e-3) / 1e9,
                             "peak": hbm, "frac": 676 * E / (total * 1e-3) / 1e9 / hbm,
                             "work": "676 B per edge over the four ops", "peak_source": "MEASURED_PEAKS.json (%s)" % peak_kind},
                "ops": per_op, "ms_sum_of_ops_timed_alone": sum(ms.values()),
                "l2": "flushed before the step (value) and before every op (ops)"}
    else:
        torch.manual_seed(2)
        n, ci, co = 1000, 32, 64
        x = torch.randn(n, ci, 16)
        v = torch.randn(n, 3)
        v = v / v.norm(dim=1, keepdim=True)
        W = torch.randn(34, ci, co) / math.sqrt(ci)
        g = torch.randn(n, co, 16)
        x, v, W, g = x.to(dev), v.to(dev), W.to(dev), g.to(dev)
        Y = _bm.spherical_harmonics(v, 3)
        ops = [("tensor_product", lambda: _bm.tensor_product(x, Y, W)),
               ("tensor_product_backward", lambda: _bm.tensor_product_backward(x, Y, W, g))]
        ms = timed_ops(ops, args.steps, args.warmup, flush)
        flops = {"tensor_product": 2.0 * 156 * ci * co * n + 2.0 * 611 * ci * n,
                 "tensor_product_backward": 2 * 2.0 * 156 * ci * co * n + 2 * 2.0 * 611 * ci * n}
        per_op = [{"op": k, "ms": ms[k], "GFLOP": flops[k] / 1e9,
                   "TFLOP/s": flops[k] / (ms[k] * 1e-3) / 1e12} for k in ms]
        total = sum(ms.values())
        line = {"metric": "config3: weighted tensor_product fwd+bwd, N=1000, C_in=32, C_out=64",
                "value": n / (total * 1e-3) / 1e6, "unit": "Msamples/s", "ms_per_step": total, "steps": args.steps,
                "warmup": args.warmup, "dtype": "f32", "data": "synthetic (seed 2)", "ops": per_op,
                "note": "latency-bound at this size: one launch of each GEMM group covers the whole problem",
                "l2": "flushed before every op"}
    line["gpu_launches"] = lib.bm_launch_count() - l0
    print(json.dumps(line), flush=True)


class ProfiledCompute:
    """GpuCompute with a launch-profiler boundary before every library call, so
    that each kernel's device time starts after the torch / NCCL work before it."""

    def __init__(self, inner, lib):
        self.inner, self.lib = inner, lib

    def neighbors(self, *a):
        self.lib.bm_profile_mark()
        return self.inner.neighbors(*a)

    def layer(self, x_l, vec, W, src, dst, graph, G_l, mark=lambda name: None):
        def mk(name):
            mark(name)
            self.lib.bm_profile_mark()
        self.lib.bm_profile_mark()
        return self.inner.layer(x_l, vec, W, src, dst, graph, G_l, mk)

    def pos_grad(self, *a):
        self.lib.bm_profile_mark()
        return self.inner.pos_grad(*a)


def run_sharded(args, world, rank, local):
    """The 1M-atom periodic system over `world` GPUs: slab decomposition with NCCL halo."""
    import ctypes
    from batmobile.distributed import SlabDecomposition, GpuCompute, StageEvents
    from batmobile._lib import lib
    cfg = CFG5
    dev = torch.device("cuda", local)
    torch.manual_seed(cfg["seed"])
    pos = torch.rand(cfg["n"], 3) * cfg["box"]
    W = (torch.randn(34, cfg["c"], cfg["c"]) / math.sqrt(cfg["c"])).to(dev)
    sd = SlabDecomposition([cfg["box"]] * 3, cfg["rc"], world, rank)
    own = torch.nonzero(sd.owned_mask(pos)).flatten()
    pos_h = pos[own].contiguous()
    gen = torch.Generator(device=dev).manual_seed(cfg["seed"] + rank)
    x = torch.randn(own.numel(), cfg["c"], 16, device=dev, generator=gen)
    G = torch.randn(own.numel(), cfg["c"], 16, device=dev, generator=gen)
    pos_d = pos_h.to(dev)
    comp = GpuCompute()
    clk = ClockSampler(local).__enter__()   # spans warm-up and the timed region (short runs)
    clk.wait_first()
    for _ in range(args.warmup):
        sd.step(comp, pos_d, x, W, G)
    torch.cuda.synchronize()
    launches0 = lib.bm_launch_count()
    times, edges = [], 0
    barrier(world)
    torch.cuda.synchronize()
    for _ in range(args.steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        _, _, _, _, edges = sd.step(comp, pos_d, x, W, G)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    clk.__exit__(None, None, None)
    barrier(world)
    launches = lib.bm_launch_count() - launches0
    t = max_over_ranks(sum(times) / len(times), world)
    e_all = torch.tensor([float(edges)], dtype=torch.float64, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(e_all)
    E = int(e_all.item())
    value = E / (t * 1e-3) / 1e6

    # per-stage device time (CUDA events between the stages, this rank; mean of 3 steps)
    stage_ms = {}
    for _ in range(3):
        ev = StageEvents()
        sd.step(comp, pos_d, x, W, G, stages=ev)
        for k, v in ev.ms().items():
            stage_ms[k] = stage_ms.get(k, 0.0) + v / 3
    # per-kernel device time (launch profiler, one step) and the dominant kernel's roofline
    lib.bm_profile_start(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _, _, _, _, e_local = sd.step(ProfiledCompute(comp, lib), pos_d, x, W, G)
    torch.cuda.synchronize()
    lib.bm_profile_stop()
    kernels = kernel_table(1)
    n_own = own.numel()
    n_local = n_own + sd.last_halo.n_from_left + sd.last_halo.n_from_right
    mma_peak = probe_mma_tf32_tflops(lib)
    peaks, peak_kind = measured_peaks()
    roofline = roofline_of(kernels, layer_work(e_local, n_own, n_local, cfg["c"]), mma_peak,
                           peaks.get("bf16_tflops", 1590.0) / 2.0, peak_kind, peaks)
    roofline["stage_ms_rank0"] = stage_ms
    roofline["limiting_stage"] = max(stage_ms, key=stage_ms.get) if stage_ms else None
    roofline["note"] = ("dominant kernel on rank 0 (library launch profiler, one step); stage_ms_rank0 = CUDA "
                        "events between the stages of the step on rank 0")

    # end to end: owned positions and features in from pinned host memory; the
    # layer output, feature gradients, forces and the weight gradient out, every step
    pos_p, x_p = pos_h.pin_memory(), x.cpu().pin_memory()
    gpos_p = torch.empty(n_own, 3).pin_memory()
    gw_p = torch.empty(34, cfg["c"], cfg["c"]).pin_memory()
    out_p = torch.empty(n_own, cfg["c"], 16).pin_memory()
    gx_p = torch.empty(n_own, cfg["c"], 16).pin_memory()
    e2e = []
    barrier(world)
    for i in range(max(2, args.steps // 2) + 1):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        pd = pos_p.to(dev, non_blocking=True)
        xd = x_p.to(dev, non_blocking=True)
        out_d, gx_d, gw, gp, _ = sd.step(comp, pd, xd, W, G)
        gpos_p.copy_(gp, non_blocking=True)
        gw_p.copy_(gw, non_blocking=True)
        out_p.copy_(out_d, non_blocking=True)
        gx_p.copy_(gx_d, non_blocking=True)
        e.record()
        e.synchronize()
        if i > 0:
            e2e.append(s.elapsed_time(e))
    t_e2e = max_over_ranks(sum(e2e) / len(e2e), world)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "Medges/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "config5: N=1,000,000 atoms, periodic cube L=259, rc=5.0, C=64, L_max=3, "
                                       "%d x-slabs, NCCL halo of ghost positions/features, reverse halo of ghost "
                                       "gradients, dW all-reduce; step = neighbour list + fused layer fwd + bwd"
                                       % world,
                           "n_atoms": cfg["n"], "edges": E, "channels": cfg["c"],
                           "parallelism": "spatial slabs x%d" % world,
                           "l2": "working set (tens of GB) exceeds L2"},
                "clocks": clk.summary(),
                "e2e": {"value": E / (t_e2e * 1e-3) / 1e6, "unit": "Medges/s", "ms_per_step": t_e2e,
                        "h2d_bytes_per_step": (pos_p.numel() + x_p.numel()) * 4,
                        "d2h_bytes_per_step": (gpos_p.numel() + gw_p.numel() + out_p.numel() + gx_p.numel()) * 4,
                        "what": "rank 0's pinned owned positions + features in; layer output, feature gradients, "
                                "forces and weight gradients out"},
                "gpu_launches": launches, "gpu_launches_per_step": launches / args.steps,
                "roofline": roofline, "kernels": kernels,
                "cpu_baseline": None}
        print(json.dumps(line), flush=True)


def e2e_pipelined(bm, _bm, lib, pos, x, W, G, pos_p, x_p, flush, args, world, E):
    """End-to-end throughput of a stream of steps through the public API, the
    way a serving or training loop runs it: two sets of device buffers and
    graphs, so that step k+1's inputs are copied in (host -> device stream) and
    step k's results copied out (device -> host stream) while the GPU computes.
    Every step copies its positions and node features in from pinned host
    memory and its layer output, feature gradients, forces and weight
    gradients out; the L2 is flushed (on the compute stream) before every
    step's graphs.  Timed from the first step's copy in to the last step's
    copy out (CUDA events), divided by the step count."""
    dev = pos.device
    sets = []
    for _ in range(2):
        pk, xk = pos.clone(), x.clone()
        st = GraphedStep(bm, _bm, lib, CFG, pk, xk, W, G)
        host = {"out": torch.empty(tuple(st.outputs[0].shape)).pin_memory(),
                "gx": torch.empty(tuple(st.outputs[1].shape)).pin_memory(),
                "gw": torch.empty(tuple(st.outputs[2].shape)).pin_memory(),
                "gpos": torch.empty(tuple(st.outputs[3].shape)).pin_memory()}
        sets.append((st, pk, xk, host))
    main = torch.cuda.current_stream()
    h2d_s, d2h_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    g_done = [None, None]    # graphs of the set's last step finished (inputs free)
    d_done = [None, None]    # copies out of the set's last step finished (outputs free)
    start = end = None
    total = args.warmup + args.steps
    barrier(world)
    torch.cuda.synchronize()
    for k in range(total):
        if k == args.warmup:
            start = torch.cuda.Event(enable_timing=True)
            start.record(main)
            h2d_s.wait_stream(main)
        i = k % 2
        st, pk, xk, host = sets[i]
        with torch.cuda.stream(h2d_s):
            if g_done[i] is not None:
                h2d_s.wait_event(g_done[i])
            pk.copy_(pos_p, non_blocking=True)
            xk.copy_(x_p, non_blocking=True)
            in_ready = torch.cuda.Event()
            in_ready.record(h2d_s)
        main.wait_event(in_ready)
        if d_done[i] is not None:
            main.wait_event(d_done[i])
        flush_l2(flush)
        out, gx, gw, gpos, _ = st()
        g_done[i] = torch.cuda.Event()
        g_done[i].record(main)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(g_done[i])
            host["out"].copy_(out, non_blocking=True)
            host["gx"].copy_(gx, non_blocking=True)
            host["gw"].copy_(gw, non_blocking=True)
            host["gpos"].copy_(gpos, non_blocking=True)
            d_done[i] = torch.cuda.Event()
            d_done[i].record(d2h_s)
    main.wait_stream(d2h_s)
    end = torch.cuda.Event(enable_timing=True)
    end.record(main)
    end.synchronize()
    for st, _, _, host in sets:
        st.check()
        for name, dv in zip(("out", "gx", "gw", "gpos"), st.outputs):   # what reached the host is the result
            if not torch.equal(host[name], dv.cpu()):
                raise RuntimeError("pipelined end-to-end step: host copy of %s differs from the device result" % name)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps, world)
    return {"value": world * E / (ms * 1e-3) / 1e6, "ms_per_step": ms,
            "what": "a stream of steps through the public API with two sets of device buffers: each step's "
                    "pinned host positions + node features copied in while the previous step computes, its layer "
                    "output, feature gradients, forces and weight gradients copied out while the next one "
                    "computes (H2D and D2H on their own streams, L2 flushed before every step); timed from the "
                    "first copy in to the last copy out"}


def trace_step(step, replays):
    """Kernel timeline of `replays` warm replays of the graphed step from a
    CUPTI trace (torch.profiler): per-kernel device time per replay, and for
    the last replay its span from the first kernel's start to the last one's
    end against the kernels' summed durations (the difference is idle time)."""
    from torch.profiler import profile, ProfilerActivity
    for _ in range(5):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(replays):
            step()
        torch.cuda.synchronize()
    evs = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
                 key=lambda e: e.time_range.start)
    per = {}
    for e in evs:
        k = e.name.split("(")[0]
        per[k] = per.get(k, 0.0) + (e.time_range.end - e.time_range.start) / replays
    firsts = [i for i, e in enumerate(evs) if "nl_bin_kernel" in e.name]
    last = evs[firsts[-1]:] if firsts else evs
    span = last[-1].time_range.end - last[0].time_range.start if last else 0.0
    busy = sum(e.time_range.end - e.time_range.start for e in last)
    print(json.dumps({"trace": "graphed 5000-atom step, %d warm replays" % replays,
                      "us_per_replay": dict(sorted(per.items(), key=lambda kv: -kv[1])),
                      "last_replay_span_us": span, "last_replay_kernels_us": busy,
                      "idle_us": span - busy}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--trace", action="store_true",
                    help="5000-atom step: CUPTI kernel timeline of warm graph replays (torch.profiler), "
                         "per-kernel device time per replay and the idle time between kernels; no bench line")
    ap.add_argument("--config", type=int, default=None, choices=[2, 3, 4, 5],
                    help="4 = single-GPU layer step (default at 1 GPU); 5 = 1M-atom sharded step (default at >1 GPU); "
                         "2 / 3 = the standalone-op workloads (SH + TP simple on 1M edges; weighted TP)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    config = args.config or (5 if world > 1 else 4)
    if config in (2, 3):
        run_ops_config(args, config)
        return
    if config == 5:
        run_sharded(args, world, rank, local)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import batmobile as bm
    from batmobile import _batmobile as _bm
    from batmobile._lib import lib

    dev = torch.device("cuda", local)
    pos_h, x_h, W_h, G_h = make_inputs(CFG)
    pos, x, W, G = (t.to(dev) for t in (pos_h, x_h, W_h, G_h))
    if args.trace:
        trace_step(GraphedStep(bm, _bm, lib, CFG, pos, x, W, G), max(args.steps, 1))
        return
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # > L2 (126 MB)

    # pinned host buffers of the end-to-end step (its graph copies the results into them)
    pin = lambda t: t.pin_memory()  # noqa: E731
    pos_p, x_p = pin(pos_h), pin(x_h)
    host = {"gpos": torch.empty(CFG["n"], 3).pin_memory(), "gw": torch.empty_like(W_h).pin_memory(),
            "out": torch.empty(CFG["n"], CFG["c"], 16).pin_memory(), "gx": torch.empty_like(x_h).pin_memory()}
    step = GraphedStep(bm, _bm, lib, CFG, pos, x, W, G, host=host)
    clk = ClockSampler(local).__enter__()  # spans warm-up and the timed region
    clk.wait_first()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident timed region: per-step events, L2 flushed between steps
    launches0 = lib.bm_launch_count()
    step_ms = []
    barrier(world)
    torch.cuda.synchronize()
    for _ in range(args.steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        out, gx, gw, gpos, E = step()
        e.record()
        e.synchronize()
        step_ms.append(s.elapsed_time(e))
    torch.cuda.synchronize()
    clk.__exit__(None, None, None)
    step.check()   # every replay's list fitted the edge buffers (outside the timed region)
    barrier(world)
    # library kernels of the two graphs per replay (eager launches, if any, on top)
    launches = lib.bm_launch_count() - launches0 + args.steps * step.launches

    # ---- per-stage device time: eager steps with events around each API call
    gpu_step(bm, _bm, pos, x, W, G, CFG)  # untimed: eager allocations outside the graph's memory pool
    torch.cuda.synchronize()
    stages = Stages()
    for _ in range(3):
        flush_l2(flush)
        gpu_step(bm, _bm, pos, x, W, G, CFG, stages)
        torch.cuda.synchronize()
        stages.collect()
    t_step = max_over_ranks(sum(step_ms) / len(step_ms), world)
    value = world * E / (t_step * 1e-3) / 1e6

    # ---- end to end through the public API: host inputs -> device -> host results;
    # the results go back on a copy stream as soon as each is final (inside the graph)
    h2d = pos_p.numel() * 4 + x_p.numel() * 4
    d2h = sum(t.numel() for t in host.values()) * 4
    e2e_ms = []
    copy_stream = torch.cuda.Stream(device=dev)
    main = torch.cuda.current_stream()
    barrier(world)
    for i in range(args.warmup + args.steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x_ready = torch.cuda.Event()
        s.record()
        pos.copy_(pos_p, non_blocking=True)
        # the 20 MB feature copy (into the graph's input buffer) overlaps the
        # neighbour list, which needs positions only
        copy_stream.wait_stream(main)
        with torch.cuda.stream(copy_stream):
            x.copy_(x_p, non_blocking=True)
            x_ready.record()
        step(x_ready=x_ready, e2e=True)
        e.record()
        e.synchronize()
        if i >= args.warmup:
            e2e_ms.append(s.elapsed_time(e))
    step.check()
    t_e2e = max_over_ranks(sum(e2e_ms) / len(e2e_ms), world)
    e2e_value = world * E / (t_e2e * 1e-3) / 1e6
    e2e_pipe = e2e_pipelined(bm, _bm, lib, pos, x, W, G, pos_p, x_p, flush, args, world, E)

    # ---- per-kernel device time (library launch profiler) and the dominant kernel's roofline
    import ctypes
    from batmobile._lib import profile_report
    nprof = 3
    lib.bm_profile_start(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    for _ in range(nprof):
        flush_l2(flush)
        lib.bm_profile_mark()
        gpu_step(bm, _bm, pos, x, W, G, CFG, lib=lib)
    lib.bm_profile_stop()
    kernels = kernel_table(nprof)
    n, c = CFG["n"], CFG["c"]
    mma_peak = probe_mma_tf32_tflops(lib)
    peaks, peak_kind = measured_peaks()
    tf32_peak = peaks.get("bf16_tflops", 1590.0) / 2.0   # dense tf32 = half the bf16 rate
    # DRAM bytes (read + write) per launch from one ncu capture of each kernel at
    # this workload (profiles/layer_edge_kernels_mma_config4_ncu.md and
    # profiles/layer_kernels_config4_ncu_full.md give the commands)
    ncu_traffic = {
        "layer_bwd(target)": 230.76e6 + 4.98e6,
        "layer_fwd(aggregate)": 31.34e6 + 148.60e6,
        "layer_bwd(source aggregate)": 29.55e6 + 147.20e6,
        "tc_gemm(mix->irreps)": 213.12e6 + 20.42e6,
    }
    roofline = roofline_of(kernels, layer_work(E, n, n, c), mma_peak, tf32_peak, peak_kind, peaks, ncu_traffic)
    roofline["traffic_unit"] = ("DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum of the "
                                "capture in profiles/, same workload)")
    stage_ms = {k: v / 3 for k, v in stages.ms.items()}
    roofline.update({
        "layer_fraction": {
            "achieved_tflops": 3 * (2.0 * 611 * c * E + 2.0 * 156 * c * c * n) /
                               ((stage_ms["layer_fwd"] + stage_ms["layer_bwd"]) * 1e-3) / 1e12,
            "note": "reference-order algorithmic work of the whole layer (3 x CG at edge granularity + 3 x mix) "
                    "over forward + backward time"},
        "stage_ms": stage_ms,
    })

    mace = mace_step_timing(bm, dev, pos, max(3, args.steps // 10), args.warmup) if world == 1 else None

    # ---- the same step with the channel mix in single-pass TF32 (inside the 2e-3
    # tolerance allowed for a tf32 mix); the headline above is the fp32-accurate 3xTF32 mix
    lib.bm_set_mix_precision(1)
    try:
        step_tf32 = GraphedStep(bm, _bm, lib, CFG, pos, x, W, G)
        for _ in range(args.warmup):
            step_tf32()
        torch.cuda.synchronize()
        tf32_ms = []
        for _ in range(max(3, args.steps // 4)):
            flush_l2(flush)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            step_tf32()
            e.record()
            e.synchronize()
            tf32_ms.append(s.elapsed_time(e))
    finally:
        lib.bm_set_mix_precision(0)
    t_tf32 = max_over_ranks(sum(tf32_ms) / len(tf32_ms), world)
    tf32_mix = {"value": world * E / (t_tf32 * 1e-3) / 1e6, "unit": "Medges/s", "ms_per_step": t_tf32,
                "steps": len(tf32_ms),
                "what": "same step, channel mixes in single-pass TF32 (about 5e-4 relative; gate 2e-3)"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import ref_ops  # noqa: F401  (CPU baseline leg only)
        ei, vec = _bm.neighbor_list(pos, [CFG["box"]] * 3, CFG["rc"])
        cpu = cpu_baseline(x_h, vec.cpu(), W_h, ei.cpu(), G_h, n, pos=pos_h, cfg=CFG)
    ref_cuda_row = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # comparison arm: the reference's own CUDA kernels, compiled for sm_100a
        # from its sources (oracle/ref_cuda.py), on the same inputs
        from oracle import ref_cuda
        ei, vec = _bm.neighbor_list(pos, [CFG["box"]] * 3, CFG["rc"])
        ref_cuda_row = ref_cuda.time_pipelines(x, vec, W, G, ei, n)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "Medges/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": t_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": WORKLOAD, "n_atoms": n, "edges": E, "channels": c,
                           "parallelism": "replicas" if world > 1 else "single",
                           "l2": "flushed (256 MB write, then read back) between timed steps"},
                "clocks": clk.summary(),
                "e2e": {"value": e2e_pipe["value"], "unit": "Medges/s", "ms_per_step": e2e_pipe["ms_per_step"],
                        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                        "what": e2e_pipe["what"],
                        "one_step_at_a_time": {
                            "value": e2e_value, "ms_per_step": t_e2e,
                            "ms_per_step_median": statistics.median(e2e_ms),
                            "ms_per_step_min_max": [min(e2e_ms), max(e2e_ms)],
                            "what": "each step alone (timed from its first copy in to its last copy out): pinned "
                                    "host positions + node features in (features on a copy stream, overlapping "
                                    "the neighbour list); layer output, feature gradients, forces and weight "
                                    "gradients out on a copy stream as each is final (the output during the "
                                    "backward, the feature gradient during the edge-gradient pass)"}},
                "gpu_launches": launches // args.steps * args.steps,
                "gpu_launches_per_step": launches / args.steps,
                "roofline": roofline, "kernels": kernels, "mace_step": mace, "tf32_mix": tf32_mix,
                "cpu_baseline": cpu, "reference_cuda_b200": ref_cuda_row}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
