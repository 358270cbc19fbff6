"""The CPU oracle against the reference's golden data (no GPU)."""
import json
import math
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, relerr

GOLDEN = os.path.join(ROOT, "tests", "golden")


def test_path_count_and_order(oracle):
    # tests/test_tensor_product.py:315-340: 34 triangle-valid (l1, l2, l_out), l <= 3
    info, ents = oracle.cg_table()
    want = [(a, b, c) for a in range(4) for b in range(4) for c in range(abs(a - b), min(a + b, 3) + 1)]
    assert [tuple(r) for r in info.tolist()] == want
    assert len(ents) == 611


def test_generated_cg_matches_reference_table(oracle):
    """The product's CG table (derived from the Racah formula by csrc/gen_cg.py)
    equals the reference's vendored table entry for entry."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("gen_cg", os.path.join(ROOT, "batmobile-evo_b200", "csrc",
                                                                         "gen_cg.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    mine = {(p, a, b, o): c for (p, a, b, o, c) in gen.table()}
    _, ents = oracle.cg_table()
    ref = {(p, a, b, o): c for (p, a, b, o, c) in ents}
    assert mine.keys() == ref.keys()
    assert max(abs(mine[k] - ref[k]) for k in ref) < 2e-7


def test_cg_orthonormal(oracle):
    # sum_{m1,m2} C[m1,m2,mo] C[m1,m2,mo'] = delta (per path), to fp32 rounding
    for (l1, l2, lo, blk) in oracle.cg_blocks():
        G = torch.einsum("abo,abq->oq", blk, blk)
        assert (G - torch.eye(2 * lo + 1, dtype=G.dtype)).abs().max() < 5e-7


def test_sh_matches_reference_python(oracle):
    d = np.load(os.path.join(GOLDEN, "sh_ref.npz"))
    v = torch.from_numpy(d["vectors"]).double()
    for L in range(5):
        assert relerr(oracle.sh(v, L), torch.from_numpy(d["Y%d" % L])) < 1e-12
    g = oracle.sh_backward(v, torch.from_numpy(d["gY3"]))
    assert relerr(g, torch.from_numpy(d["gv3"])) < 1e-12


@pytest.mark.parametrize("L", range(7))
def test_sh_gram_identity(oracle, L):
    # tests/test_spherical_harmonics.py:176-203: Fibonacci sphere, mean Y Y^T = I
    n = 20000
    i = torch.arange(n, dtype=torch.float64) + 0.5
    phi = torch.acos(1 - 2 * i / n)
    th = math.pi * (1 + 5 ** 0.5) * i
    P = torch.stack([torch.sin(phi) * torch.cos(th), torch.sin(phi) * torch.sin(th), torch.cos(phi)], 1)
    Y = oracle.sh(P, L)
    G = Y.T @ Y / n
    assert (G - torch.eye((L + 1) ** 2, dtype=G.dtype)).abs().max() < 1e-4
    assert torch.all(Y[:, 0] == 1)


def _rotation(seed):
    g = torch.Generator().manual_seed(seed)
    q, r = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=torch.float64))
    q = q * torch.sign(torch.diagonal(r))
    if torch.det(q) < 0:
        q[:, 0] = -q[:, 0]
    return q


def _wigner(oracle, R, L=3):
    """D(R) in the SH basis: least squares of Y(R v) = D Y(v)."""
    g = torch.Generator().manual_seed(7)
    v = torch.randn(400, 3, generator=g, dtype=torch.float64)
    v = v / v.norm(dim=1, keepdim=True)
    Y, YR = oracle.sh(v, L), oracle.sh(v @ R.T, L)
    return torch.linalg.lstsq(Y, YR).solution.T


def test_tp_equivariant(oracle):
    """TP(D x, D y) = D TP(x, y) for the weighted product (oracle self-consistency
    of the CG table with the SH basis)."""
    R = _rotation(3)
    D = _wigner(oracle, R)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, 4, 16, generator=g, dtype=torch.float64)
    y = torch.randn(5, 16, generator=g, dtype=torch.float64)
    W = torch.randn(34, 4, 3, generator=g, dtype=torch.float64)
    lhs = oracle.tp(x @ D.T, y @ D.T, W)
    rhs = oracle.tp(x, y, W) @ D.T
    assert relerr(lhs, rhs) < 1e-6  # table is fp32-rounded


def test_nl_oracle_matches_reference_bruteforce(oracle):
    d = np.load(os.path.join(GOLDEN, "nl_ref.npz"))
    for n in (100, 300):
        pos = torch.from_numpy(d["pos%d" % n])
        box = float(d["box%d" % n])
        ei, vec = oracle.nl_bruteforce(pos, [box] * 3, 5.0)
        assert torch.equal(ei, torch.from_numpy(d["ei%d" % n]).long())
        assert torch.equal(vec, torch.from_numpy(d["vec%d" % n]))
        ei2, vec2 = oracle.nl_cells(pos, [box] * 3, 5.0)
        assert torch.equal(ei2, ei) and torch.equal(vec2, vec)


def test_nl_cells_matches_bruteforce_noncubic(oracle):
    g = torch.Generator().manual_seed(11)
    box = [23.0, 17.5, 31.25]
    pos = torch.rand(1500, 3, generator=g) * torch.tensor(box) + torch.tensor([0.0, -20.0, 40.0])
    for sl in (False, True):
        a = oracle.nl_bruteforce(pos, box, 4.5, self_loops=sl)
        b = oracle.nl_cells(pos, box, 4.5, self_loops=sl)
        assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_csr_oracle(oracle):
    ei = torch.tensor([[0, 1, 2, 3, 0], [1, 1, 0, 2, 2]])
    rp, col = oracle.edge_index_to_csr(ei, 4)
    assert rp.tolist() == [0, 1, 3, 5, 5]
    assert col.tolist() == [2, 0, 1, 3, 4]


def test_layer_oracle_is_chain_of_ops(oracle):
    """interaction() equals SH -> gather -> tp -> index_add done by hand, and the
    chunked version equals the unchunked one."""
    g = torch.Generator().manual_seed(5)
    n, e, c = 12, 40, 3
    x = torch.randn(n, c, 16, generator=g, dtype=torch.float64)
    v = torch.randn(e, 3, generator=g, dtype=torch.float64)
    W = torch.randn(34, c, 2, generator=g, dtype=torch.float64)
    ei = torch.randint(0, n, (2, e), generator=g)
    a = oracle.interaction(x, v, W, ei, n)
    b = oracle.interaction_chunked(x, v, W, ei, n, chunk=7)
    assert relerr(a, b) < 1e-12
    Y = oracle.sh(v / v.norm(dim=1, keepdim=True), 3)
    m = oracle.tp(x[ei[0]], Y, W)
    ref = torch.zeros(n, 2, 16, dtype=torch.float64).index_add_(0, ei[1], m)
    assert relerr(a, ref) < 1e-12


TRICLINIC_CELLS = [
    [[20.0, 0.0, 0.0], [4.0, 18.0, 0.0], [-3.0, 5.0, 22.0]],    # moderate tilts
    [[16.0, 0.0, 0.0], [7.5, 15.0, 0.0], [7.0, 7.0, 14.0]],     # tilts near half a vector
    [[11.0, 0.5, 0.0], [-2.0, 10.5, 1.0], [1.5, -2.5, 12.0]],   # small: 3 bins per direction
]


def _triclinic_positions(cell, n, seed):
    g = torch.Generator().manual_seed(seed)
    s = torch.rand(n, 3, generator=g)
    s[::5] += torch.randint(-2, 3, (len(s[::5]), 3), generator=g).float()  # images outside the cell
    return (s.double() @ torch.tensor(cell, dtype=torch.float64)).float()


@pytest.mark.parametrize("ci", range(len(TRICLINIC_CELLS)))
def test_nl_triclinic_oracle_is_minimum_image(oracle, ci):
    """The triclinic oracle (fractional rounding, fp32) against a float64 search of
    all 125 nearby images: every pair clearly inside the cutoff is an edge with the
    shortest image vector, every pair clearly outside is not (pairs within 1e-4 of
    the cutoff may go either way in fp32)."""
    cell = TRICLINIC_CELLS[ci]
    rc = 4.5
    pos = _triclinic_positions(cell, 400, ci)
    ei, vec = oracle.nl_bruteforce_cell(pos, cell, rc)
    H = torch.tensor(cell, dtype=torch.float64)
    p = pos.double() @ torch.linalg.inv(H)
    p = (p - torch.floor(p)) @ H  # wrapped into the cell, so 5^3 images cover every minimum
    shifts = torch.stack(torch.meshgrid(*[torch.arange(-2, 3)] * 3, indexing="ij"), -1).reshape(-1, 3).double() @ H
    d = (p.unsqueeze(0) - p.unsqueeze(1)).unsqueeze(2) + shifts  # [i, j, image, 3] = p_j - p_i + shift
    r = d.norm(dim=-1)
    rmin, kmin = r.min(dim=2)
    rmin.fill_diagonal_(float("inf"))
    inside = rmin < rc * (1 - 1e-4)
    outside = rmin > rc * (1 + 1e-4)
    got = torch.zeros_like(inside)
    got[ei[0], ei[1]] = True
    assert bool((got & inside).sum() == inside.sum())
    assert not bool((got & outside).any())
    best = d[ei[0], ei[1], kmin[ei[0], ei[1]]]
    assert float((vec.double() - best).abs().max()) < 1e-4
    # antisymmetric: the reverse of every edge is an edge with the negated vector
    key = ei[0] * 400 + ei[1]
    rkey = ei[1] * 400 + ei[0]
    order = torch.argsort(key)
    idx = order[torch.searchsorted(key[order], rkey)]
    assert torch.equal(key[idx], rkey)
    assert torch.equal(vec[idx], -vec)


def test_nl_triclinic_oracle_diagonal_cell(oracle):
    """A diagonal cell through the fractional-coordinate predicate gives the
    orthorhombic edge set (away from the cutoff boundary)."""
    box = [19.0, 23.5, 21.0]
    pos = torch.rand(500, 3, generator=torch.Generator().manual_seed(7)) * torch.tensor(box)
    a, _ = oracle.nl_bruteforce(pos, box, 5.0)
    b, _ = oracle.nl_bruteforce_cell(pos, torch.diag(torch.tensor(box)).tolist(), 5.0)
    sa = set(map(tuple, a.T.tolist()))
    sb = set(map(tuple, b.T.tolist()))
    diff = sa ^ sb
    for i, j in diff:  # only boundary pairs may differ
        d = pos[j].double() - pos[i].double()
        L = torch.tensor(box, dtype=torch.float64)
        d = d - torch.round(d / L) * L
        assert abs(float(d.norm()) - 5.0) < 1e-4


def test_hoisted_interaction_equals_reference_form(oracle):
    """The reordered float64 checker used at the headline sizes (edge-summed
    outer products, then CG and the channel mix once per atom) equals the
    reference's per-edge formulation, forward and gradients, to float64 rounding."""
    g = torch.Generator().manual_seed(7)
    n, box, ci, co = 150, 13.0, 6, 5
    pos = torch.rand(n, 3, generator=g) * box
    ei, vec = oracle.nl_bruteforce(pos, [box] * 3, 5.0)
    x = torch.randn(n, ci, 16, generator=g, dtype=torch.float64)
    W = torch.randn(34, ci, co, generator=g, dtype=torch.float64)
    v = vec.double()
    a = oracle.interaction(x, v, W, ei, n)
    b = oracle.interaction_hoisted(x, v, W, ei, n, chunk=500)
    assert relerr(b, a) < 1e-12
    go = torch.randn(a.shape, generator=g, dtype=torch.float64)
    ra = oracle.grads(lambda p, q, r: oracle.interaction(p, q, r, ei, n), [x, v, W], go)
    rb = oracle.grads(lambda p, q, r: oracle.interaction_hoisted(p, q, r, ei, n, chunk=500), [x, v, W], go)
    for u, w in zip(rb, ra):
        assert relerr(u, w) < 1e-12
