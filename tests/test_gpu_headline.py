"""Parity at the benchmarked sizes, through the exact code path bench.py times.

* The interaction-layer step at N=5000 atoms (periodic cube L=44.3, rc=5,
  ~151k edges), C=64, seed 3, inputs drawn exactly as bench.make_inputs draws
  them, run through bench.GraphedStep (neighbour-list plan, symmetric CSR
  views, CUDA-graph replays, node features copied in on a side stream): edge
  set bit-exact against the C cell-list oracle; layer output and gradients
  w.r.t. node features, weights and positions against the float64 oracle
  (reordered form, itself checked against the per-edge reference form in
  tests/test_oracle_golden.py, plus a direct per-edge spot check here).
* The message pass of the 1000-atom CPU-reference workload (seed 0, L=29.7,
  C=32) against the per-edge reference formulation.
* The 1M-atom periodic neighbour list (seed 4, L=259) bit-exact against the
  C cell-list oracle.
Tolerance: max|gpu - ref| / max|ref| <= 1e-5 (fp32-accurate 3xTF32 mixes)."""
import math
import os

import pytest
import torch

from conftest import relerr

pytestmark = pytest.mark.gpu
TOL = 1e-5
dev = "cuda"


@pytest.fixture(scope="module")
def bench_mod():
    import bench
    return bench


def test_graphed_step_at_benchmark_size_matches_oracle(bm, oracle, bench_mod):
    from batmobile import _batmobile as _bm
    from batmobile._lib import lib
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = bench_mod.CFG
    n = cfg["n"]
    pos_h, x_h, W_h, G_h = bench_mod.make_inputs(cfg)
    pos, x, W, G = (t.to(dev) for t in (pos_h, x_h, W_h, G_h))
    host = {"gpos": torch.empty(n, 3).pin_memory(), "gw": torch.empty_like(W_h).pin_memory(),
            "out": torch.empty(n, cfg["c"], 16).pin_memory(), "gx": torch.empty_like(x_h).pin_memory()}
    step = bench_mod.GraphedStep(bm, _bm, lib, cfg, pos, x, W, G, host=host)
    out, gx, gw, gpos, E = (t.clone() if torch.is_tensor(t) else t for t in step())
    # a second replay with the features copied in from pinned memory on a side
    # stream (the end-to-end path) gives the same bits
    x.zero_()
    side = torch.cuda.Stream()
    ready = torch.cuda.Event()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        x.copy_(x_h.pin_memory(), non_blocking=True)
        ready.record()
    out2, gx2, gw2, gpos2, E2 = step(x_ready=ready)
    torch.cuda.synchronize()
    assert E2 == E
    for a, b in ((out, out2), (gx, gx2), (gw, gw2), (gpos, gpos2)):
        assert torch.equal(a, b)
    # the end-to-end graph: the same kernels, results streamed into pinned host memory
    for t in host.values():
        t.fill_(float("nan"))
    step(x_ready=None, e2e=True)
    torch.cuda.synchronize()
    for a, k in ((out, "out"), (gx, "gx"), (gw, "gw"), (gpos, "gpos")):
        assert torch.equal(a.cpu(), host[k])

    step.check()   # the list fitted the step's edge buffers, no device wait timed out
    rei, rvec = oracle.nl_cells(pos_h, [cfg["box"]] * 3, cfg["rc"])
    assert E == rei.shape[1] == step.edges()
    assert torch.equal(step.ei[:, :E].cpu(), rei) and torch.equal(step.vec[:E].cpu(), rvec)

    xd, vd, Wd = x_h.double(), rvec.double(), W_h.double()
    f = lambda a, b, c: oracle.interaction_hoisted(a, b, c, rei, n)  # noqa: E731
    ref = f(xd, vd, Wd)
    assert relerr(out, ref) < TOL
    rx, rv, rw = oracle.grads(f, [xd, vd, Wd], G_h.double())
    assert relerr(gx, rx) < TOL
    assert relerr(gw, rw) < TOL
    # forces: v_e = p[dst] - p[src] (minimum image), so dpos = in-sum - out-sum of dv
    rp = torch.zeros(n, 3, dtype=torch.float64).index_add_(0, rei[1], rv).index_add_(0, rei[0], -rv)
    assert relerr(gpos, rp) < TOL

    # direct spot check against the per-edge reference form on 200 targets' edges
    mask = rei[1] < 200
    sub = oracle.interaction(xd, vd[mask], Wd, rei[:, mask], n)[:200]
    assert relerr(out[:200], sub) < TOL


def test_message_pass_cpu_reference_workload_seed0(bm, oracle):
    torch.manual_seed(0)
    n, box, c = 1000, 29.7, 32
    pos = torch.rand(n, 3) * box
    ei, vec = bm.neighbor_list(pos.to(dev), [box] * 3, 5.0)
    rei, rvec = oracle.nl_bruteforce(pos, [box] * 3, 5.0)
    assert torch.equal(ei.cpu(), rei) and torch.equal(vec.cpu(), rvec)
    x = torch.randn(n, c, 16)
    W = torch.randn(34, c, c) / math.sqrt(c)
    xg, vg, Wg = (t.to(dev).requires_grad_(True) for t in (x, vec.cpu(), W))
    out = bm.fused_tp_scatter(xg, vg, Wg, edge_index=ei)
    f = lambda a, b, w: oracle.interaction(a, b, w, rei, n)  # noqa: E731
    ref = f(x.double(), rvec.double(), W.double())
    assert relerr(out, ref) < TOL
    go = torch.randn(out.shape, generator=torch.Generator().manual_seed(1))
    gx, gv, gw = torch.autograd.grad(out, [xg, vg, Wg], go.to(dev))
    rx, rv, rw = oracle.grads(f, [x.double(), rvec.double(), W.double()], go.double())
    assert relerr(gx, rx) < TOL and relerr(gv, rv) < TOL and relerr(gw, rw) < TOL


def test_neighbor_list_1m_atoms_bit_exact(bm, oracle):
    torch.manual_seed(4)
    n, box = 1_000_000, 259.0
    pos = torch.rand(n, 3) * box
    ei, vec = bm.neighbor_list(pos.to(dev), [box] * 3, 5.0)
    rei, rvec = oracle.nl_cells(pos, [box] * 3, 5.0)
    assert ei.shape == rei.shape
    assert torch.equal(ei.cpu(), rei)
    assert torch.equal(vec.cpu(), rvec)
