"""Graph kernels and the neighbour list on the GPU against the oracle.

Neighbour list: bit-exact edge set, order and vectors.  Float outputs:
max|gpu - ref| / max|ref| <= 1e-5 against float64.
"""
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, relerr

pytestmark = pytest.mark.gpu
TOL = 1e-5
dev = "cuda"


def graph(n, e, seed):
    g = torch.Generator().manual_seed(seed)
    ei = torch.randint(0, n, (2, e), generator=g)
    v = torch.randn(e, 3, generator=g)
    v = v / v.norm(dim=1, keepdim=True)
    return ei, v


def test_edge_index_to_csr(bm, oracle):
    ei, _ = graph(500, 12000, 1)
    rp, col = bm.edge_index_to_csr(ei.to(dev), 500)
    rrp, rcol = oracle.edge_index_to_csr(ei, 500)
    assert torch.equal(rp.cpu(), rrp) and torch.equal(col.cpu(), rcol)
    # atoms with no incoming edges, and a hub
    ei2 = torch.cat([ei, torch.stack([torch.arange(3000) % 500, torch.full((3000,), 7)])], 1)
    ei2[1][ei2[1] == 3] = 4
    rp, col = bm.edge_index_to_csr(ei2.to(dev), 600)
    rrp, rcol = oracle.edge_index_to_csr(ei2, 600)
    assert torch.equal(rp.cpu(), rrp) and torch.equal(col.cpu(), rcol)


def test_fused_sh_tp_simple(bm, oracle):
    ei, v = graph(300, 5000, 2)
    x = torch.randn(300, 24, 16, generator=torch.Generator().manual_seed(3))
    got = bm.fused_sh_tp_simple(v.to(dev), x.to(dev), ei[0].to(dev))
    assert relerr(got, oracle.fused_sh_tp_simple(v.double(), x.double(), ei[0])) < TOL


def test_fused_message_passing_simple(bm, oracle):
    ei, v = graph(300, 5000, 4)
    x = torch.randn(300, 16, 16, generator=torch.Generator().manual_seed(5))
    rp, col = bm.edge_index_to_csr(ei.to(dev), 300)
    got = bm.fused_message_passing_simple(x.to(dev), v.to(dev), ei.to(dev), rp, col)
    assert relerr(got, oracle.fused_mp_simple(x.double(), v.double(), ei, 300)) < TOL
    # unfused path of benchmarks/benchmark_fused_sh_tp.py:34-61 with the same kernels
    msg = bm.fused_sh_tp_simple(v.to(dev), x.to(dev), ei[0].to(dev))
    unf = torch.zeros(300, 16, 16, device=dev).index_add_(0, ei[1].to(dev), msg)
    assert relerr(got, unf.double()) < TOL


def test_fused_message_passing_weighted(bm, oracle):
    ei, v = graph(200, 3000, 6)
    rp, col = oracle.edge_index_to_csr(ei, 200)
    src_csr = ei[0][col]                     # binding contract: sources in CSR order
    v_csr = v[col]
    x = torch.randn(200, 8, 16, generator=torch.Generator().manual_seed(7))
    W2 = torch.randn(8, 12, generator=torch.Generator().manual_seed(8))
    got = bm.fused_message_passing(x.to(dev), v_csr.to(dev), W2.to(dev), rp.to(dev), src_csr.to(dev))
    ref = oracle.fused_mp_weighted(x.double(), v_csr.double(), W2.double(), rp, src_csr)
    assert relerr(got, ref) < TOL


def test_neighbor_list_reference_golden(bm):
    d = np.load(os.path.join(ROOT, "tests", "golden", "nl_ref.npz"))
    for n in (100, 300):
        pos = torch.from_numpy(d["pos%d" % n]).to(dev)
        box = float(d["box%d" % n])
        ei, vec = bm.neighbor_list(pos, torch.eye(3) * box, 5.0)
        assert torch.equal(ei.cpu(), torch.from_numpy(d["ei%d" % n]).long())
        assert torch.equal(vec.cpu(), torch.from_numpy(d["vec%d" % n]))


@pytest.mark.parametrize("n,box,rc,self_loops", [
    (1000, 29.7, 5.0, False),      # 1000 atoms, ~20 neighbours
    (5000, 44.3, 5.0, False),      # 5000 atoms, ~30 neighbours
    (2000, [23.0, 17.5, 31.25], 4.5, True),
    (64, 9.0, 5.0, False),         # box < 2 rc: 3 cells per axis, min-image
    (1, 10.0, 3.0, True),
])
def test_neighbor_list_bit_exact(bm, oracle, n, box, rc, self_loops):
    g = torch.Generator().manual_seed(n)
    b = torch.tensor(box if isinstance(box, list) else [box] * 3)
    pos = torch.rand(n, 3, generator=g) * b
    pos[::7] -= b * 1.5  # some atoms outside the primary cell
    ei, vec = bm.neighbor_list(pos.to(dev), b, rc, self_loops=self_loops)
    rei, rvec = oracle.nl_cells(pos, b.tolist(), rc, self_loops)
    assert torch.equal(ei.cpu(), rei)
    assert torch.equal(vec.cpu(), rvec)


def test_neighbor_list_empty_and_deterministic(bm):
    ei, vec = bm.neighbor_list(torch.zeros(0, 3, device=dev), [10.0, 10.0, 10.0], 2.0)
    assert ei.shape == (2, 0) and vec.shape == (0, 3)
    pos = (torch.rand(3000, 3, generator=torch.Generator().manual_seed(9)) * 30).to(dev)
    a = bm.neighbor_list(pos, [30.0] * 3, 4.0)
    b = bm.neighbor_list(pos, [30.0] * 3, 4.0)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_neighbor_list_reference_ctypes_abi(bm):
    """neighbor_list_cuda / neighbor_list_free with the reference's struct (int32 edges)."""
    import ctypes
    from batmobile._lib import lib, NeighborListResult
    pos = (torch.rand(800, 3, generator=torch.Generator().manual_seed(10)) * 25).to(dev)
    cell = (torch.eye(3) * 25).to(dev)
    res = NeighborListResult()
    err = lib.neighbor_list_cuda(ctypes.c_void_p(pos.data_ptr()), ctypes.c_void_p(cell.data_ptr()), 800,
                                 ctypes.c_float(5.0), False, ctypes.byref(res), None)
    assert err == 0
    E = res.num_edges
    ei, vec = bm.neighbor_list(pos, [25.0] * 3, 5.0)
    assert E == ei.shape[1]
    got = torch.empty(2 * E, dtype=torch.int32, device=dev)
    gv = torch.empty(E * 3, dtype=torch.float32, device=dev)
    cudart = ctypes.CDLL("libcudart.so.12")
    cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    assert cudart.cudaMemcpy(got.data_ptr(), res.edge_index, 8 * E, 3) == 0
    assert cudart.cudaMemcpy(gv.data_ptr(), res.edge_vectors, 12 * E, 3) == 0
    lib.neighbor_list_free(ctypes.byref(res))
    assert torch.equal(got.view(2, E).long(), ei)
    assert torch.equal(gv.view(E, 3), vec)


def test_neighbor_list_1m_properties(bm):
    """1M atoms, L=259: symmetric edge set, count ~30 per atom, vectors within rc."""
    g = torch.Generator().manual_seed(4)
    pos = (torch.rand(1_000_000, 3, generator=g) * 259.0).to(dev)
    ei, vec, rp = bm.neighbor_list(pos, [259.0] * 3, 5.0, return_row_ptr=True)
    E = ei.shape[1]
    assert 25 < E / 1e6 < 35
    assert bool((vec.norm(dim=1) <= 5.0 + 1e-5).all())
    assert bool((ei[0][1:] >= ei[0][:-1]).all())
    key = ei[0] * 1_000_000 + ei[1]
    rkey = ei[1] * 1_000_000 + ei[0]
    assert torch.equal(torch.sort(key).values, torch.sort(rkey).values)
    assert torch.equal(rp[1:] - rp[:-1], torch.bincount(ei[0], minlength=1_000_000))


def test_csr_reverse_matches_sorted_csr(bm):
    """The symmetric fast path: csr_reverse on a full neighbour list equals the
    target-grouped CSR built by counting and sorting, and is an involution;
    a layer step on the resulting EdgeGraph matches the generic one bit for bit."""
    from batmobile import _batmobile as _bm
    g = torch.Generator().manual_seed(11)
    n, box = 600, 22.0
    pos = (torch.rand(n, 3, generator=g) * box).to(dev)
    ei, vec, rp = _bm.neighbor_list(pos, [box] * 3, 5.0, return_row_ptr=True)
    rev = _bm.csr_reverse(rp, ei[1].contiguous())
    rp2, perm2 = _bm.edge_index_to_csr(ei, n)
    assert torch.equal(rp2, rp)
    assert torch.equal(perm2, rev)
    assert torch.equal(rev[rev], torch.arange(ei.shape[1], device=dev))
    x = torch.randn(n, 8, 16, generator=g).to(dev)
    W = (torch.randn(34, 8, 8, generator=g) / 8 ** 0.5).to(dev)
    ga = bm.EdgeGraph(ei, n, src_row_ptr=rp)
    gb = bm.EdgeGraph(ei, n, src_row_ptr=rp, symmetric=True)
    oa, _ = _bm.layer_forward(x, vec, W, ga.src, ga.row_ptr_dst, ga.perm_dst)
    ob, _ = _bm.layer_forward(x, vec, W, gb.src, gb.row_ptr_dst, gb.perm_dst)
    assert torch.equal(oa, ob)
    assert lib_error_free()


def lib_error_free():
    from batmobile._lib import lib
    return lib.bm_device_error_check() == 0


TRICLINIC_CELLS = [
    ([[20.0, 0.0, 0.0], [4.0, 18.0, 0.0], [-3.0, 5.0, 22.0]], 1500, 5.0, False),
    ([[16.0, 0.0, 0.0], [7.5, 15.0, 0.0], [7.0, 7.0, 14.0]], 1200, 4.5, True),
    ([[11.0, 0.5, 0.0], [-2.0, 10.5, 1.0], [1.5, -2.5, 12.0]], 400, 4.0, False),  # 3 bins per direction
    ([[30.0, 0.0, 0.0], [0.0, 28.0, 0.0], [0.0, 0.0, 33.0]], 2000, 5.0, False),  # diagonal [3,3]: orthorhombic
]


@pytest.mark.parametrize("ci", range(len(TRICLINIC_CELLS)))
def test_neighbor_list_triclinic_bit_exact(bm, oracle, ci):
    """General cells: edge set, order and vectors equal the fractional-coordinate
    brute force bit for bit; the list stays exactly symmetric, so the
    reverse-edge CSR equals the sorted target CSR."""
    from batmobile import _batmobile as _bm
    cell, n, rc, self_loops = TRICLINIC_CELLS[ci]
    g = torch.Generator().manual_seed(100 + ci)
    s = torch.rand(n, 3, generator=g)
    s[::5] += torch.randint(-2, 3, (len(s[::5]), 3), generator=g).float()
    pos = (s.double() @ torch.tensor(cell, dtype=torch.float64)).float()
    ei, vec, rp = _bm.neighbor_list(pos.to(dev), torch.tensor(cell), rc, self_loops=self_loops, return_row_ptr=True)
    if ci == 3:
        rei, rvec = oracle.nl_cells(pos, [cell[0][0], cell[1][1], cell[2][2]], rc, self_loops)
    else:
        rei, rvec = oracle.nl_bruteforce_cell(pos, cell, rc, self_loops)
    assert ei.shape[1] > 0
    assert torch.equal(ei.cpu(), rei)
    assert torch.equal(vec.cpu(), rvec)
    if not self_loops:
        rev = _bm.csr_reverse(rp, ei[1].contiguous())
        rp2, perm2 = _bm.edge_index_to_csr(ei, n)
        assert torch.equal(rp2, rp)
        assert torch.equal(perm2, rev)
    # row-restricted variant: the first rows are a prefix of the full list
    k = n // 3
    ei_k, vec_k = _bm.neighbor_list(pos.to(dev), torch.tensor(cell), rc, self_loops=self_loops, n_rows=k)
    m = int((rei[0] < k).sum())
    assert torch.equal(ei_k.cpu(), rei[:, :m])
    assert torch.equal(vec_k.cpu(), rvec[:m])
    assert lib_error_free()


def test_neighbor_list_triclinic_rejects_degenerate_cell(bm):
    pos = torch.rand(10, 3, device=dev)
    with pytest.raises(RuntimeError, match="linearly dependent"):
        bm.neighbor_list(pos, [[5.0, 0.0, 0.0], [10.0, 0.0, 0.0], [0.0, 0.0, 5.0]], 1.0)


def test_neighbor_list_plan_graph_replay(bm):
    """NeighborListPlan: count captured in a CUDA graph and replayed after the
    positions change gives the same edges as the one-call neighbour list."""
    from batmobile import _batmobile as _bm
    g = torch.Generator().manual_seed(31)
    n, box, rc = 2000, 30.0, 4.5
    pos = (torch.rand(n, 3, generator=g) * box).to(dev)
    plan = _bm.NeighborListPlan(pos, [box] * 3, rc)
    plan.count()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        plan.count()
    pos.copy_((torch.rand(n, 3, generator=g) * box).to(dev))  # new positions, same buffer
    graph.replay()
    e = plan.num_edges()
    ei = torch.empty(2, e, dtype=torch.int64, device=dev)
    vec = torch.empty(e, 3, device=dev)
    plan.fill(ei, vec)
    rei, rvec, rrp = _bm.neighbor_list(pos.clone(), [box] * 3, rc, return_row_ptr=True)
    assert torch.equal(ei, rei) and torch.equal(vec, rvec) and torch.equal(plan.row_ptr, rrp)
    assert lib_error_free()


def test_neighbor_list_fill_short_buffers_flagged_not_overrun(bm):
    """A fill given fewer edge slots than the count found writes nothing past
    them and reports BM_ERR_CAPACITY through the device error flag."""
    from batmobile import _batmobile as _bm
    from batmobile._lib import lib
    g = torch.Generator().manual_seed(9)
    n, box = 600, 18.0
    pos = (torch.rand(n, 3, generator=g) * box).to(dev)
    plan = _bm.NeighborListPlan(pos, [box] * 3, 5.0)
    plan.count()
    E = plan.num_edges()
    short, guard = E - 37, 4096
    ei_buf = torch.full((2 * short + guard,), -7, dtype=torch.int64, device=dev)
    vec_buf = torch.full((short + guard, 3), -7.0, dtype=torch.float32, device=dev)
    plan.fill(ei_buf[:2 * short].view(2, short), vec_buf[:short])
    torch.cuda.synchronize()
    assert lib.bm_device_error_check() == 4          # BM_ERR_CAPACITY
    assert lib.bm_device_error_check() == 0          # read and cleared
    assert bool((ei_buf[2 * short:] == -7).all()) and bool((vec_buf[short:] == -7.0).all())
    # a full-size fill afterwards is complete and exact
    ei, vec = bm.neighbor_list(pos, [box] * 3, 5.0)
    assert ei.shape[1] == E
