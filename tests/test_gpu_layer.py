"""Fused SH -> weighted TP -> scatter layer against the reference formulation
(normalise -> SH -> x[src] -> tensor_product -> index_add, float64 autograd).
Tolerance: max|gpu - ref| / max|ref| <= 1e-5 (fp32)."""
import pytest
import torch

from conftest import relerr

pytestmark = pytest.mark.gpu
TOL = 1e-5
dev = "cuda"


def pbc_system(n, box, rc, ci, co, seed):
    g = torch.Generator().manual_seed(seed)
    pos = torch.rand(n, 3, generator=g) * box
    x = torch.randn(n, ci, 16, generator=g)
    W = torch.randn(34, ci, co, generator=g) / ci ** 0.5
    return pos, x, W


@pytest.mark.parametrize("n,box,ci,co", [(200, 15.0, 16, 16), (1000, 29.7, 32, 32), (300, 18.0, 70, 20),
                                         (500, 10.0, 7, 9), (160, 12.0, 33, 5)])
def test_layer_forward_backward(bm, oracle, n, box, ci, co):
    """Includes odd channel counts and, at 500 atoms in a 10 A box, atoms with
    more than 250 incoming edges."""
    pos, x, W = pbc_system(n, box, 5.0, ci, co, n)
    ei, vec = bm.neighbor_list(pos.to(dev), [box] * 3, 5.0)
    xg = x.to(dev).requires_grad_(True)
    vg = vec.clone().requires_grad_(True)
    Wg = W.to(dev).requires_grad_(True)
    out = bm.fused_tp_scatter(xg, vg, Wg, edge_index=ei)
    ref = oracle.interaction(x.double(), vec.double().cpu(), W.double(), ei.cpu(), n)
    assert relerr(out, ref) < TOL
    go = torch.randn(out.shape, generator=torch.Generator().manual_seed(1)).to(dev)
    gx, gv, gw = torch.autograd.grad(out, [xg, vg, Wg], go)
    rx, rv, rw = oracle.grads(lambda a, b, c: oracle.interaction(a, b, c, ei.cpu(), n),
                              [x.double(), vec.double().cpu(), W.double()], go.double().cpu())
    assert relerr(gx, rx) < TOL
    assert relerr(gv, rv) < TOL
    assert relerr(gw, rw) < TOL


def test_layer_tf32_mix_within_gate(bm, oracle):
    """Single-pass TF32 channel mixes (bm_set_mix_precision(1)): the fused layer's
    output and gradients stay inside the 2e-3 tolerance allowed for a tf32 mix."""
    from batmobile._lib import lib
    n, box, ci, co = 1000, 29.7, 64, 64
    pos, x, W = pbc_system(n, box, 5.0, ci, co, 21)
    ei, vec = bm.neighbor_list(pos.to(dev), [box] * 3, 5.0)
    ref = oracle.interaction(x.double(), vec.double().cpu(), W.double(), ei.cpu(), n)
    go = torch.randn(ref.shape, generator=torch.Generator().manual_seed(2))
    rx, rv, rw = oracle.grads(lambda a, b, c: oracle.interaction(a, b, c, ei.cpu(), n),
                              [x.double(), vec.double().cpu(), W.double()], go.double())
    assert lib.bm_set_mix_precision(1) == 0
    try:
        xg, vg, Wg = (t.to(dev).requires_grad_(True) for t in (x, vec.cpu(), W))
        out = bm.fused_tp_scatter(xg, vg, Wg, edge_index=ei)
        gx, gv, gw = torch.autograd.grad(out, [xg, vg, Wg], go.to(dev))
    finally:
        lib.bm_set_mix_precision(0)
    for got, want in ((out, ref), (gx, rx), (gv, rv), (gw, rw)):
        assert relerr(got, want) < 2e-3


def test_layer_general_graph_with_isolated_atoms(bm, oracle):
    """Random (non-symmetric) edges, atoms without edges, zero-length vectors."""
    g = torch.Generator().manual_seed(3)
    n, e = 150, 2500
    ei = torch.randint(0, n - 10, (2, e), generator=g)
    v = torch.randn(e, 3, generator=g)
    v[5] = 0.0
    x = torch.randn(n, 8, 16, generator=g)
    W = torch.randn(34, 8, 12, generator=g)
    xg, vg, Wg = (t.to(dev).requires_grad_(True) for t in (x, v, W))
    out = bm.fused_tp_scatter(xg, vg, Wg, edge_index=ei.to(dev))
    ref = oracle.interaction(x.double(), v.double(), W.double(), ei, n)
    assert relerr(out, ref) < TOL
    assert float(out[n - 10:].abs().max()) == 0.0
    go = torch.randn(out.shape, generator=g).to(dev)
    gx, gv, gw = torch.autograd.grad(out, [xg, vg, Wg], go)
    rx, rv, rw = oracle.grads(lambda a, b, c: oracle.interaction(a, b, c, ei, n),
                              [x.double(), v.double(), W.double()], go.double().cpu())
    assert relerr(gx, rx) < TOL and relerr(gv, rv) < TOL and relerr(gw, rw) < TOL


def test_forces_through_edge_vectors(bm, oracle):
    """d(sum out * g)/d(pos) via the NL vectors and the deterministic edge -> atom reduction."""
    n, box = 400, 20.0
    pos, x, W = pbc_system(n, box, 5.0, 8, 8, 11)
    ei, _ = bm.neighbor_list(pos.to(dev), [box] * 3, 5.0)
    graph = bm.EdgeGraph(ei, n)
    boxt = torch.full((3,), box, device=dev)
    pg = pos.to(dev).requires_grad_(True)
    v = bm.EdgeVectorsFunction.apply(pg, boxt, graph)
    out = bm.fused_tp_scatter(x.to(dev), v, W.to(dev), graph=graph)
    go = torch.randn(out.shape, generator=torch.Generator().manual_seed(2)).to(dev)
    (gp,) = torch.autograd.grad(out, [pg], go)

    def f(p):
        d = p[ei[1].cpu()] - p[ei[0].cpu()]
        d = d - torch.round(d / box) * box
        return oracle.interaction(x.double(), d, W.double(), ei.cpu(), n)

    (rp,) = oracle.grads(f, [pos.double()], go.double().cpu())
    assert relerr(gp, rp) < TOL


def test_layer_config4_properties(bm):
    """5000 atoms, C=64 (the benchmarked size): linearity in W, determinism, and the sum rule
    sum_n out = sum_e msg (checked through the unfused kernels)."""
    g = torch.Generator().manual_seed(3)
    n, box = 5000, 44.3
    pos = (torch.rand(n, 3, generator=g) * box).to(dev)
    x = torch.randn(n, 64, 16, generator=g).to(dev)
    W1 = (torch.randn(34, 64, 64, generator=g) / 8).to(dev)
    W2 = (torch.randn(34, 64, 64, generator=g) / 8).to(dev)
    ei, vec = bm.neighbor_list(pos, [box] * 3, 5.0)
    graph = bm.EdgeGraph(ei, n)
    a = bm.fused_tp_scatter(x, vec, W1, graph=graph)
    b = bm.fused_tp_scatter(x, vec, W2, graph=graph)
    c = bm.fused_tp_scatter(x, vec, W1 + 2 * W2, graph=graph)
    assert relerr(c, a + 2 * b) < 1e-5
    assert torch.equal(a, bm.fused_tp_scatter(x, vec, W1, graph=graph))
    # against the unfused chain built from this library's own kernels
    Y = bm.spherical_harmonics(vec / vec.norm(dim=1, keepdim=True).clamp(min=1e-8), 3)
    out = torch.zeros_like(a)
    for s in range(0, ei.shape[1], 20000):
        sl = slice(s, s + 20000)
        out.index_add_(0, ei[1, sl], bm.tensor_product(x[ei[0, sl]].contiguous(), Y[sl].contiguous(), W1))
    assert relerr(a, out.double()) < 1e-5


@pytest.mark.parametrize("n,box,ci,co,k", [(200, 15.0, 16, 16, 2), (120, 13.0, 8, 12, 3), (60, 10.0, 70, 8, 2)])
def test_layer_radial_weights(bm, oracle, n, box, ci, co, k):
    """Per-edge weights W_e = sum_k R[e, k] W[k] (the radial weight net's last
    linear layer): forward and gradients w.r.t. x, edge vectors, R and W."""
    pos, x, _ = pbc_system(n, box, 5.0, ci, co, n + 7)
    g = torch.Generator().manual_seed(n + 8)
    W = torch.randn(k, 34, ci, co, generator=g) / ci ** 0.5
    ei, vec = bm.neighbor_list(pos.to(dev), [box] * 3, 5.0)
    R = torch.randn(ei.shape[1], k, generator=g)
    xg = x.to(dev).requires_grad_(True)
    vg = vec.clone().requires_grad_(True)
    Rg = R.to(dev).requires_grad_(True)
    Wg = W.to(dev).requires_grad_(True)
    out = bm.fused_tp_scatter_radial(xg, vg, Rg, Wg, edge_index=ei)

    def ref(a, b, r, w):
        eic = ei.cpu()
        Y = oracle.sh(oracle.unit(b, 1e-8), 3)
        o = torch.zeros(n, co, 16, dtype=a.dtype)
        for j in range(k):
            o.index_add_(0, eic[1], r[:, j, None, None] * oracle.tp(a[eic[0]], Y, w[j]))
        return o

    rin = [x.double(), vec.double().cpu(), R.double(), W.double()]
    assert relerr(out, ref(*rin)) < TOL
    go = torch.randn(out.shape, generator=torch.Generator().manual_seed(2)).to(dev)
    got = torch.autograd.grad(out, [xg, vg, Rg, Wg], go)
    exp = oracle.grads(ref, rin, go.double().cpu())
    for a, b in zip(got, exp):
        assert relerr(a, b) < TOL


def test_layer_target_subset_matches_full(bm):
    """n_targets: the first T atoms are the only targets, all N atoms are sources
    (the owned-first layout of a spatial domain).  Results equal the full-N pass
    on a graph whose rows >= T are empty with a zero upstream gradient there."""
    from batmobile import _batmobile as _bm
    g = torch.Generator().manual_seed(17)
    n, t, e, ci, co = 700, 420, 9000, 32, 24
    src = torch.randint(0, n, (e,), generator=g)
    dst = torch.randint(0, t, (e,), generator=g)
    ei = torch.stack([src, dst]).to(dev)
    v = torch.randn(e, 3, generator=g).to(dev)
    x = torch.randn(n, ci, 16, generator=g).to(dev)
    W = (torch.randn(34, ci, co, generator=g) / ci ** 0.5).to(dev)
    G = torch.randn(t, co, 16, generator=g).to(dev)
    graph = bm.EdgeGraph(ei, n)
    rps, ps = graph.src_csr
    full, slots = _bm.layer_forward(x, v, W, graph.src, graph.row_ptr_dst, graph.perm_dst)
    Gf = torch.cat([G, torch.zeros(n - t, co, 16, device=dev)], 0)
    fgx, fgv, fgw = _bm.layer_backward(x, v, W, graph.src, graph.dst, graph.row_ptr_dst, graph.perm_dst, rps, ps,
                                       slots, Gf)
    rpt = graph.row_ptr_dst[:t + 1]
    out, slots_t = _bm.layer_forward(x, v, W, graph.src, rpt, graph.perm_dst, n_targets=t)
    gx, gv, gw = _bm.layer_backward(x, v, W, graph.src, graph.dst, rpt, graph.perm_dst, rps, ps, slots_t, G,
                                    n_targets=t)
    assert out.shape == (t, co, 16) and gx.shape == x.shape
    assert torch.equal(out, full[:t])
    assert relerr(gx, fgx) < 1e-6 and relerr(gv, fgv) < 1e-6 and relerr(gw, fgw) < 1e-6


def test_gpu_compute_owned_targets_matches_full(bm):
    """The sharded step's local compute (batmobile.distributed.GpuCompute) on one
    GPU: owned atoms first and the only targets, every other atom a ghost source.
    Output, gradients and forces equal the whole-system layer with the upstream
    gradient zero outside the owned atoms."""
    from batmobile import _batmobile as _bm
    from batmobile.distributed import GpuCompute
    g = torch.Generator().manual_seed(23)
    n, box, rc, c = 1500, 26.0, 5.0, 16
    pos = torch.rand(n, 3, generator=g) * box
    x = torch.randn(n, c, 16, generator=g)
    W = torch.randn(34, c, c, generator=g) / 4
    G = torch.randn(n, c, 16, generator=g)
    owned = pos[:, 0] < box / 2
    order = torch.cat([torch.nonzero(owned).flatten(), torch.nonzero(~owned).flatten()])
    n_own = int(owned.sum())
    comp = GpuCompute()
    pos_l, x_l = pos[order].to(dev), x[order].to(dev)
    G_l = G[order].to(dev)
    G_l[n_own:] = 0
    src, dst, vec, graph = comp.neighbors(pos_l, n_own, [box] * 3, rc)
    out, gx, gv, gw = comp.layer(x_l, vec, W.to(dev), src, dst, graph, G_l[:n_own].contiguous())
    gp = comp.pos_grad(gv, src, dst, graph, n)
    Gm = G.clone()
    Gm[~owned] = 0
    ei, rvec, rp = _bm.neighbor_list(pos.to(dev), [box] * 3, rc, return_row_ptr=True)
    eg = bm.EdgeGraph(ei, n, src_row_ptr=rp)
    ref, slots = _bm.layer_forward(x.to(dev), rvec, W.to(dev), eg.src, eg.row_ptr_dst, eg.perm_dst)
    rps, ps = eg.src_csr
    rgx, rgv, rgw = _bm.layer_backward(x.to(dev), rvec, W.to(dev), eg.src, eg.dst, eg.row_ptr_dst, eg.perm_dst,
                                       rps, ps, slots, Gm.to(dev))
    rgp = _bm.edge_grad_to_pos(rgv, eg.row_ptr_dst, eg.perm_dst, rps, ps)
    od = order.to(dev)
    assert out.shape[0] == n_own
    assert relerr(out, ref[od[:n_own]]) < 1e-6
    assert relerr(gx, rgx[od]) < 1e-6 and relerr(gw, rgw) < 1e-6
    assert relerr(gp, rgp[od]) < 1e-5

