"""CPU oracle: a restatement of the reference's own PyTorch formulation of the
hot path.  TEST INFRASTRUCTURE ONLY -- imported by tests/, by
__graft_entry__.smoke() as the checker and by bench.py's CPU-baseline leg.  The
product (batmobile-evo_b200/) never imports it.

Every function cites the reference file:line it restates (paths inside the
batmobile-evo tree).  Arithmetic is torch on the CPU, float64 by default for
the checker; fp32 when used as the timed CPU baseline.

Parity pins:
 * CG table: tests/golden/cg_l3.json is parsed from the reference's vendored
   include/cg_coefficients_l3.cuh by tests/golden/gen_golden.py; the oracle
   uses exactly those 611 coefficients.
 * SH l <= 4 and its backward: tests/golden/sh_ref.npz was produced by running
   the reference's python/batmobile/autograd.py functions.  l = 5, 6 follow the
   reference CUDA kernel (src/spherical_harmonics/spherical_harmonics.cu:152-256)
   because the reference's Python fallback for l >= 5 is not orthonormal; they
   are pinned by the Fibonacci-sphere Gram test of
   tests/test_spherical_harmonics.py:176-203.
 * Neighbour list: pinned against the reference's own CPU brute force
   (tests/test_neighbor_list.cu:30-68) compiled into oracle/_ref.
"""
import json
import math
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(os.path.dirname(HERE), "tests", "golden")

# ------------------------------------------------------------- CG table --

_CG = None


def cg_table():
    """(path_info [34,3], entries list of (path, m1, m2, mo, c)) from the golden
    copy of include/cg_coefficients_l3.cuh:23-792 (flat 0..15 irreps indices)."""
    global _CG
    if _CG is None:
        with open(os.path.join(GOLDEN, "cg_l3.json")) as f:
            d = json.load(f)
        info = d["block_info"]  # [l1, l2, lo, off1, off2, offo]
        ents = []
        for p, (b, e) in enumerate(d["block_ranges"]):
            l1, l2, lo, o1, o2, oo = info[p]
            for k in range(b, e):
                m1, m2, mo = d["entry_info"][k]
                ents.append((p, o1 + m1, o2 + m2, oo + mo, d["coeffs"][k]))
        _CG = (np.array([r[:3] for r in info], dtype=np.int32), ents)
    return _CG


def cg_blocks(dtype=torch.float64):
    """Per path: (l1, l2, lo, dense block [2l1+1, 2l2+1, 2lo+1]) as in
    tests/test_tensor_product.py:230-246 (cg = sqrt(2lo+1) * w3j)."""
    info, ents = cg_table()
    blocks = []
    for p in range(34):
        l1, l2, lo = (int(x) for x in info[p])
        blocks.append([l1, l2, lo, torch.zeros(2 * l1 + 1, 2 * l2 + 1, 2 * lo + 1, dtype=dtype)])
    for (p, m1, m2, mo, c) in ents:
        l1, l2, lo, blk = blocks[p]
        blk[m1 - l1 * l1, m2 - l2 * l2, mo - lo * lo] = c
    return [tuple(b) for b in blocks]


def cg_dense(dtype=torch.float64):
    """All 611 entries as a dense [16, 16, 16] tensor C[m1, m2, mo]."""
    _, ents = cg_table()
    C = torch.zeros(16, 16, 16, dtype=dtype)
    for (p, m1, m2, mo, c) in ents:
        C[m1, m2, mo] += c
    return C


# --------------------------------------------------- spherical harmonics --

def sh(vectors, lmax):
    """Real SH, component normalisation.  l <= 3: python/batmobile/autograd.py:296-341;
    l = 4..6: src/spherical_harmonics/spherical_harmonics.cu:99-256."""
    x, y, z = vectors[:, 0], vectors[:, 1], vectors[:, 2]
    out = [torch.ones_like(x)]
    if lmax >= 1:
        c1 = 1.7320508075688772
        out += [c1 * x, c1 * y, c1 * z]
    if lmax >= 2:
        s15, s5 = 3.872983346207417, 2.23606797749979
        x2, y2, z2 = x * x, y * y, z * z
        x2z2 = x2 + z2
        out += [s15 * x * z, s15 * x * y, s5 * (y2 - 0.5 * x2z2), s15 * y * z, 0.5 * s15 * (z2 - x2)]
    if lmax >= 3:
        c30, c31, c32, c33 = 1.0801234497346432, 2.6457513110645907, 1.6201851746019651, 1.3228756555322954
        s20, s24 = out[4], out[8]
        out += [c30 * (s20 * z + s24 * x), c31 * s20 * y, c32 * (4 * y2 - x2z2) * x,
                c33 * y * (2 * y2 - 3 * x2z2), c32 * z * (4 * y2 - x2z2), c31 * s24 * y,
                c30 * (s24 * z - s20 * x)]
    if lmax >= 4:
        a = out[9:16]
        out += [
            1.0606601717798214 * (a[0] * z + a[6] * x),
            0.75 * a[0] * y + 0.9185586535436917 * a[1] * z + 0.9185586535436917 * a[5] * x,
            -0.2004459314343183 * a[0] * z + 0.9819805060619656 * a[1] * y + 0.7763237542601484 * a[2] * z
            + 0.7763237542601484 * a[4] * x + 0.2004459314343183 * a[6] * x,
            -0.3471825374147068 * a[1] * z + 1.0978875820670997 * a[2] * y + 0.8964214570007952 * a[3] * x
            + 0.3471825374147068 * a[5] * x,
            -0.6943650748294136 * a[2] * x + 1.1338934190276817 * a[3] * y - 0.6943650748294136 * a[4] * z,
            -0.3471825374147068 * a[1] * x + 0.8964214570007952 * a[3] * z + 1.0978875820670997 * a[4] * y
            - 0.3471825374147068 * a[5] * z,
            -0.2004459314343183 * a[0] * x - 0.7763237542601484 * a[2] * x + 0.7763237542601484 * a[4] * z
            + 0.9819805060619656 * a[5] * y - 0.2004459314343183 * a[6] * z,
            -0.9185586535436917 * a[1] * x + 0.9185586535436917 * a[5] * z + 0.75 * a[6] * y,
            1.0606601717798214 * (-a[0] * x + a[6] * z),
        ]
    if lmax >= 5:
        a = out[16:25]
        out += [
            1.0488088481701516 * (a[0] * z + a[8] * x),
            0.6633249580710801 * a[0] * y + 0.9380831519646859 * a[1] * z + 0.9380831519646859 * a[7] * x,
            -0.1563471919941143 * a[0] * z + 0.8844332774281066 * a[1] * y + 0.8273115763993905 * a[2] * z
            + 0.8273115763993905 * a[6] * x + 0.1563471919941143 * a[8] * x,
            -0.2708012801545320 * a[1] * z + 1.0132456102380443 * a[2] * y + 0.7164728420068226 * a[3] * z
            + 0.7164728420068226 * a[5] * x + 0.2708012801545320 * a[7] * x,
            -0.3829708431025353 * a[2] * z + 1.0832051206181281 * a[3] * y + 0.8563488385776753 * a[4] * x
            + 0.3829708431025353 * a[6] * x,
            -0.6992058987801010 * a[3] * x + 1.1055415967851332 * a[4] * y - 0.6992058987801010 * a[5] * z,
            -0.3829708431025353 * a[2] * x + 0.8563488385776753 * a[4] * z + 1.0832051206181281 * a[5] * y
            - 0.3829708431025353 * a[6] * z,
            -0.2708012801545320 * a[1] * x - 0.7164728420068226 * a[3] * x + 0.7164728420068226 * a[5] * z
            + 1.0132456102380443 * a[6] * y - 0.2708012801545320 * a[7] * z,
            -0.1563471919941143 * a[0] * x - 0.8273115763993905 * a[2] * x + 0.8273115763993905 * a[6] * z
            + 0.8844332774281066 * a[7] * y - 0.1563471919941143 * a[8] * z,
            -0.9380831519646859 * a[1] * x + 0.9380831519646859 * a[7] * z + 0.6633249580710801 * a[8] * y,
            1.0488088481701516 * (-a[0] * x + a[8] * z),
        ]
    if lmax >= 6:
        a = out[25:36]
        out += [
            1.0408329997330663 * (a[0] * z + a[10] * x),
            0.6009252125773314 * a[0] * y + 0.9501461875826149 * a[1] * z + 0.9501461875826149 * a[9] * x,
            -0.1281176857976346 * a[0] * z + 0.8102873913406630 * a[1] * y + 0.1281176857976346 * a[10] * x
            + 0.8594395636904107 * a[2] * z + 0.8594395636904107 * a[8] * x,
            -0.2219063411496486 * a[1] * z + 0.9414688716912718 * a[2] * y + 0.7687061147858074 * a[3] * z
            + 0.7687061147858074 * a[7] * x + 0.2219063411496486 * a[9] * x,
            -0.3138229572304240 * a[2] * z + 1.0249414863810766 * a[3] * y + 0.6779350703393059 * a[4] * z
            + 0.6779350703393059 * a[6] * x + 0.3138229572304240 * a[8] * x,
            -0.4051436956703315 * a[3] * z + 1.0719094639893330 * a[4] * y + 0.8302975005345611 * a[5] * x
            + 0.4051436956703315 * a[7] * x,
            -0.7017294652672371 * a[4] * x + 1.0871146130092180 * a[5] * y - 0.7017294652672371 * a[6] * z,
            -0.4051436956703315 * a[3] * x + 0.8302975005345611 * a[5] * z + 1.0719094639893330 * a[6] * y
            - 0.4051436956703315 * a[7] * z,
            -0.3138229572304240 * a[2] * x - 0.6779350703393059 * a[4] * x + 0.6779350703393059 * a[6] * z
            + 1.0249414863810766 * a[7] * y - 0.3138229572304240 * a[8] * z,
            -0.2219063411496486 * a[1] * x - 0.7687061147858074 * a[3] * x + 0.7687061147858074 * a[7] * z
            + 0.9414688716912718 * a[8] * y - 0.2219063411496486 * a[9] * z,
            -0.1281176857976346 * a[0] * x - 0.1281176857976346 * a[10] * z - 0.8594395636904107 * a[2] * x
            + 0.8594395636904107 * a[8] * z + 0.8102873913406630 * a[9] * y,
            -0.9501461875826149 * a[1] * x + 0.6009252125773314 * a[10] * y + 0.9501461875826149 * a[9] * z,
            1.0408329997330663 * (-a[0] * x + a[10] * z),
        ]
    return torch.stack(out, dim=-1)


def sh_backward(vectors, grad_Y):
    """sum_lm g_lm dY_lm/d(x,y,z), l <= 3 (python/batmobile/autograd.py:97-281),
    evaluated by autograd through sh() (the reference's analytic form agrees to
    rounding; the golden fixture pins it)."""
    L = int(round(math.sqrt(grad_Y.shape[1]))) - 1
    if L == 0:
        return torch.zeros_like(vectors)
    v = vectors.detach().clone().requires_grad_(True)
    Y = sh(v, L)
    (g,) = torch.autograd.grad(Y, v, grad_Y)
    return g


def unit(v, eps):
    """v / max(|v|, eps) (benchmarks/benchmark_e2e_mace.py:328-329)."""
    return v / torch.linalg.norm(v, dim=-1, keepdim=True).clamp(min=eps)


# --------------------------------------------------------- tensor products --

def tp_simple(a, b):
    """out[m_o] = sum c a[m1] b[m2] over all paths with weight 1
    (src/tensor_product/tensor_product.cu:29-50)."""
    C = cg_dense(a.dtype)
    return torch.einsum("na,nb,abo->no", a, b, C)


def tp(x, Y, W):
    """Per-path einsum of tests/test_tensor_product.py:230-282:
    prod = sum_{m1,m2} cg x[n,ci,m1] Y[n,m2];  out += einsum('ncm,co->nom', prod, W[p])."""
    n, ci, _ = x.shape
    co = W.shape[2]
    out = torch.zeros(n, co, 16, dtype=x.dtype)
    for p, (l1, l2, lo, cg) in enumerate(cg_blocks(x.dtype)):
        i1 = x[:, :, l1 * l1:l1 * l1 + 2 * l1 + 1]
        i2 = Y[:, l2 * l2:l2 * l2 + 2 * l2 + 1]
        prod = torch.einsum("ncm,nk,mko->nco", i1, i2, cg)
        out[:, :, lo * lo:lo * lo + 2 * lo + 1] += torch.einsum("ncm,co->nom", prod, W[p])
    return out


def grads(fn, inputs, grad_out):
    """Vector-Jacobian product of fn at inputs (float64 autograd)."""
    ins = [t.detach().clone().requires_grad_(True) for t in inputs]
    out = fn(*ins)
    return torch.autograd.grad(out, ins, grad_out, allow_unused=True)


# ------------------------------------------------------------------ graph --

def edge_index_to_csr(edge_index, n_atoms):
    """COO -> CSR by target, col_idx = original edge ids
    (src/message_passing/fused_message_passing.cu:74-165), rows in ascending id."""
    dst = edge_index[1]
    order = torch.argsort(dst * (edge_index.shape[1] + 1) + torch.arange(dst.numel()), stable=True)
    counts = torch.bincount(dst, minlength=n_atoms)
    row_ptr = torch.zeros(n_atoms + 1, dtype=torch.int64)
    row_ptr[1:] = torch.cumsum(counts, 0)
    return row_ptr, order


def fused_sh_tp_simple(v, x, src):
    """messages[e, c] = TP_simple(x[src[e], c], Y(v[e])) (src/message_passing/fused_sh_tp.cu:73-123)."""
    Y = sh(v, 3)
    C = cg_dense(x.dtype)
    return torch.einsum("eca,eb,abo->eco", x[src], Y, C)


def fused_mp_simple(x, v, edge_index, n_atoms):
    """out[n] = sum_{e: dst=n} TP_simple(x[src e], Y(v_e))
    (src/message_passing/fused_message_passing.cu:174-255; benchmarks/benchmark_fused_sh_tp.py:34-61)."""
    msg = fused_sh_tp_simple(v, x, edge_index[0])
    out = torch.zeros(n_atoms, x.shape[1], 16, dtype=x.dtype)
    out.index_add_(0, edge_index[1], msg)
    return out


def fused_mp_weighted(x, v_csr, W2, row_ptr, col_src):
    """Binding contract of python/bindings.cpp:494-550: CSR slot k of row n has
    source col_src[k] and vector v_csr[k]; one [Ci, Co] weight for every path."""
    n = row_ptr.numel() - 1
    dst = torch.repeat_interleave(torch.arange(n), row_ptr[1:] - row_ptr[:-1])
    msg = fused_sh_tp_simple(v_csr, x, col_src)                 # [E, Ci, 16]
    agg = torch.zeros(n, x.shape[1], 16, dtype=x.dtype).index_add_(0, dst, msg)
    return torch.einsum("nim,io->nom", agg, W2)


def interaction(x, v, W, edge_index, n_atoms, eps=1e-8):
    """BatteriesInteractionBlock.forward minus the Linear
    (benchmarks/benchmark_e2e_mace.py:323-350): normalise, SH, gather x[src],
    weighted TP, scatter-add to dst."""
    Y = sh(unit(v, eps), 3)
    msg = tp(x[edge_index[0]], Y, W)
    out = torch.zeros(n_atoms, W.shape[2], 16, dtype=x.dtype)
    out.index_add_(0, edge_index[1], msg)
    return out


def interaction_chunked(x, v, W, edge_index, n_atoms, chunk=8192, eps=1e-8):
    """interaction() with the edge dimension processed in chunks to bound memory."""
    out = torch.zeros(n_atoms, W.shape[2], 16, dtype=x.dtype)
    E = v.shape[0]
    for s in range(0, E, chunk):
        ei = edge_index[:, s:s + chunk]
        Y = sh(unit(v[s:s + chunk], eps), 3)
        out.index_add_(0, ei[1], tp(x[ei[0]], Y, W))
    return out


def interaction_hoisted(x, v, W, edge_index, n_atoms, chunk=4096, eps=1e-8):
    """interaction() with the sums reordered for large systems (float64 checker):
    B[n, ci, m1, m2] = sum_{e: dst=n} x[src e, ci, m1] Y_e[m2], then per path
    out[n, co, lo] += sum_ci W[p, ci, co] sum_{m1, m2} cg[m1, m2, lo] B[n, ci, m1, m2].
    Equal in exact arithmetic to the per-edge form of
    benchmarks/benchmark_e2e_mace.py:323-350 (W does not depend on the edge and
    the TP is linear in x (x) Y); tests/test_oracle_golden.py checks the two
    agree, with gradients, to float64 rounding.  Differentiable by autograd."""
    ci = x.shape[1]
    E = v.shape[0]
    B = torch.zeros(n_atoms, ci * 16, 16, dtype=x.dtype)
    for s in range(0, E, chunk):
        ei = edge_index[:, s:s + chunk]
        Y = sh(unit(v[s:s + chunk], eps), 3)
        xs = x[ei[0]].reshape(-1, ci * 16)
        B = B.index_add(0, ei[1], xs.unsqueeze(2) * Y.unsqueeze(1))
    B = B.reshape(n_atoms, ci, 16, 16)
    out = torch.zeros(n_atoms, W.shape[2], 16, dtype=x.dtype)
    for p, (l1, l2, lo, cg) in enumerate(cg_blocks(x.dtype)):
        blk = B[:, :, l1 * l1:l1 * l1 + 2 * l1 + 1, l2 * l2:l2 * l2 + 2 * l2 + 1]
        prod = torch.einsum("ncab,abo->nco", blk, cg)
        out[:, :, lo * lo:lo * lo + 2 * lo + 1] += torch.einsum("nco,cd->ndo", prod, W[p])
    return out


# --------------------------------------------------------- neighbour list --

def nl_bruteforce(positions, box, cutoff, self_loops=False):
    """Brute-force PBC pairs of benchmarks/benchmark_neighbor_list_standalone.py:110-125
    in float32: diff = p_i - p_j; diff -= round(diff / L) * L; keep sum(diff^2) <= rc^2;
    edges in lexicographic (i, j) order.  Returns (edge_index [2,E], vectors p_j - p_i)."""
    p = positions.to(torch.float32)
    L = torch.as_tensor(box, dtype=torch.float32).reshape(3)
    diff = p.unsqueeze(1) - p.unsqueeze(0)
    diff = diff - torch.round(diff / L) * L
    d2 = (diff[..., 0] * diff[..., 0] + diff[..., 1] * diff[..., 1]) + diff[..., 2] * diff[..., 2]
    mask = d2 <= np.float32(cutoff * cutoff)
    if not self_loops:
        mask.fill_diagonal_(False)
    ei = mask.nonzero(as_tuple=False).T.contiguous()
    vec = -diff[ei[0], ei[1]]
    return ei.to(torch.int64), vec


def cell_inverse_f32(cell):
    """Hinv = inverse(H) in float64 rounded to float32 (H row-major, rows = lattice
    vectors): the inverse the triclinic neighbour list computes on the host."""
    h = np.asarray(cell, dtype=np.float32).reshape(3, 3).astype(np.float64)
    return np.linalg.inv(h).astype(np.float32)


def _rowvec3(x, y, z, M, k):
    # (x, y, z) M component k, summed left to right, every product rounded in float32
    return (x * float(M[0, k]) + y * float(M[1, k])) + z * float(M[2, k])


def min_image_tri(d, H, Hi):
    """Fractional-coordinate minimum image of Cartesian differences d [..., 3]
    (float32): s = d Hinv; s -= round(s); d = s H."""
    x, y, z = d[..., 0], d[..., 1], d[..., 2]
    s = [_rowvec3(x, y, z, Hi, k) for k in range(3)]
    s = [sk - torch.round(sk) for sk in s]
    return torch.stack([_rowvec3(s[0], s[1], s[2], H, k) for k in range(3)], dim=-1)


def nl_bruteforce_cell(positions, cell, cutoff, self_loops=False):
    """Brute-force pairs for a general (triclinic) cell, float32: the predicate of
    nl_bruteforce with the minimum image in fractional coordinates.  The reference
    reads only the cell diagonal (src/neighbor_list/neighbor_list.cu:260-267), so
    this extends its brute-force check (benchmarks/benchmark_neighbor_list_standalone.py:110-125)
    to any cell.  Returns (edge_index [2,E], vectors p_j - p_i)."""
    p = positions.to(torch.float32)
    H = np.asarray(cell, dtype=np.float32).reshape(3, 3)
    Hi = cell_inverse_f32(H)
    diff = min_image_tri(p.unsqueeze(1) - p.unsqueeze(0), H, Hi)
    d2 = (diff[..., 0] * diff[..., 0] + diff[..., 1] * diff[..., 1]) + diff[..., 2] * diff[..., 2]
    mask = d2 <= np.float32(cutoff * cutoff)
    if not self_loops:
        mask.fill_diagonal_(False)
    ei = mask.nonzero(as_tuple=False).T.contiguous()
    vec = -diff[ei[0], ei[1]]
    return ei.to(torch.int64), vec


def nl_cells(positions, box, cutoff, self_loops=False):
    """Same predicate through the C cell list oracle/nl_cells.c (large N)."""
    from . import _native
    return _native.nl_cells(positions, box, cutoff, self_loops)
