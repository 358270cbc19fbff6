"""Spherical harmonics and tensor products on the GPU against the CPU oracle.

Tolerance: max|gpu - ref| / max|ref| <= 1e-5 (fp32 paths), ref in float64.
"""
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, relerr

pytestmark = pytest.mark.gpu
TOL = 1e-5
dev = "cuda"


def unit(n, seed):
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(n, 3, generator=g)
    return v / v.norm(dim=1, keepdim=True)


@pytest.mark.parametrize("L", range(7))
def test_sh_forward(bm, oracle, L):
    v = unit(4097, 1)
    got = bm.spherical_harmonics(v.to(dev), L)
    assert got.shape == (4097, (L + 1) ** 2)
    assert relerr(got, oracle.sh(v.double(), L)) < TOL


def test_sh_golden_and_special_vectors(bm):
    d = np.load(os.path.join(ROOT, "tests", "golden", "sh_ref.npz"))
    v = torch.from_numpy(d["vectors"]).to(dev)
    for L in range(5):
        assert relerr(bm.spherical_harmonics(v, L), torch.from_numpy(d["Y%d" % L])) < TOL
    g = bm.spherical_harmonics_backward(v, torch.from_numpy(d["gY3"]).float().to(dev))
    assert relerr(g, torch.from_numpy(d["gv3"])) < TOL


def test_sh_inplace_empty_unaligned(bm, oracle):
    v = unit(1000, 2).to(dev)
    Y = torch.empty(1000, 16, device=dev)
    bm.spherical_harmonics_inplace(v, Y, 3)
    assert torch.equal(Y, bm.spherical_harmonics(v, 3))
    assert bm.spherical_harmonics(torch.empty(0, 3, device=dev), 3).shape == (0, 16)
    # input slice that is not 16-byte aligned takes the scalar staging path
    big = unit(1001, 3).to(dev)
    sl = big[1:]
    assert relerr(bm.spherical_harmonics(sl.contiguous(), 3), oracle.sh(sl.double().cpu(), 3)) < TOL
    flat = torch.cat([torch.zeros(1, device=dev), big.reshape(-1)])[1:].view(1001, 3)
    assert relerr(bm.spherical_harmonics(flat, 3), oracle.sh(big.double().cpu(), 3)) < TOL


@pytest.mark.parametrize("L", range(7))
def test_sh_backward(bm, oracle, L):
    v = unit(3001, 4)
    g = torch.randn(3001, (L + 1) ** 2, generator=torch.Generator().manual_seed(5))
    got = bm.spherical_harmonics_backward(v.to(dev), g.to(dev))
    assert relerr(got, oracle.sh_backward(v.double(), g.double())) < TOL


def test_sh_backward_high_l_autograd(bm, oracle):
    """l = 4..6 backward (the reference stops at 3): the autograd Function
    with normalisation against float64 autograd through the oracle."""
    for L in (4, 5, 6):
        v = (torch.randn(300, 3, generator=torch.Generator().manual_seed(L)) * 2).to(dev).requires_grad_(True)
        Y = bm.SphericalHarmonics.apply(v, L, True)
        g = torch.randn(Y.shape, generator=torch.Generator().manual_seed(10 + L)).to(dev)
        (gv,) = torch.autograd.grad(Y, v, g)
        vd = v.detach().double().cpu().requires_grad_(True)
        Yd = oracle.sh(oracle.unit(vd, 1e-10), L)
        (rv,) = torch.autograd.grad(Yd, vd, g.double().cpu())
        assert relerr(gv, rv) < TOL


def test_sh_autograd_normalize(bm, oracle):
    v = (torch.randn(500, 3, generator=torch.Generator().manual_seed(6)) * 3).to(dev).requires_grad_(True)
    Y = bm.spherical_harmonics_autograd(v, 3, True)
    g = torch.randn_like(Y)
    (gv,) = torch.autograd.grad(Y, v, g)
    ref = oracle.grads(lambda t: oracle.sh(t / t.norm(dim=1, keepdim=True).clamp(min=1e-10), 3),
                       [v.detach().double().cpu()], g.double().cpu())[0]
    assert relerr(gv, ref) < TOL


def test_tp_simple_forward_backward(bm, oracle):
    g = torch.Generator().manual_seed(1)
    a = torch.randn(20001, 16, generator=g)
    b = torch.randn(20001, 16, generator=g)
    go = torch.randn(20001, 16, generator=g)
    out = bm.tensor_product_simple(a.to(dev), b.to(dev))
    assert relerr(out, oracle.tp_simple(a.double(), b.double())) < TOL
    ga, gb = bm.tensor_product_simple_backward(a.to(dev), b.to(dev), go.to(dev))
    ra, rb = oracle.grads(oracle.tp_simple, [a.double(), b.double()], go.double())
    assert relerr(ga, ra) < TOL and relerr(gb, rb) < TOL


def _unaligned(t):
    """The same values at an address 4 bytes past a 16-byte boundary."""
    flat = torch.empty(t.numel() + 1, device=t.device, dtype=t.dtype)
    flat[1:] = t.reshape(-1)
    return flat[1:].view(t.shape)


@pytest.mark.parametrize("E", [1, 3, 127, 128, 129, 1000, 300001])
def test_streaming_tile_edges(bm, oracle, E):
    """The persistent TMA-staged L = 3 kernels at ragged tile ends (128-edge
    tiles, several tiles per CTA at the larger sizes): SH forward and backward
    equal the per-block kernels (taken for unaligned inputs) bit for bit; the
    simple tensor product matches the oracle."""
    g = torch.Generator().manual_seed(E)
    v = unit(E, E).to(dev)
    Y = bm.spherical_harmonics(v, 3)
    assert torch.equal(Y, bm.spherical_harmonics(_unaligned(v), 3))
    gY = torch.randn(E, 16, generator=g).to(dev)
    gv = bm.spherical_harmonics_backward(v, gY)
    assert torch.equal(gv, bm.spherical_harmonics_backward(_unaligned(v), gY))
    if E <= 1000:
        assert relerr(Y, oracle.sh(v.double().cpu(), 3)) < TOL
        assert relerr(gv, oracle.sh_backward(v.double().cpu(), gY.double().cpu())) < TOL
    a, b, go = (torch.randn(E, 16, generator=g) for _ in range(3))
    out = bm.tensor_product_simple(a.to(dev), b.to(dev))
    assert relerr(out, oracle.tp_simple(a.double(), b.double())) < TOL
    ga, gb = bm.tensor_product_simple_backward(a.to(dev), b.to(dev), go.to(dev))
    if E <= 1000:
        ra, rb = oracle.grads(oracle.tp_simple, [a.double(), b.double()], go.double())
        assert relerr(ga, ra) < TOL and relerr(gb, rb) < TOL
    else:   # linearity of each gradient in the upstream gradient and the other operand
        ga2, _ = bm.tensor_product_simple_backward(a.to(dev), b.to(dev), (2 * go).to(dev))
        assert torch.equal(ga2, 2 * ga)
        _, gb_ = bm.tensor_product_simple_backward(a.to(dev), b.to(dev), go.to(dev))
        assert torch.equal(gb_, gb)
        ref_gb = oracle.grads(oracle.tp_simple, [a[:2000].double(), b[:2000].double()], go[:2000].double())[1]
        assert relerr(gb[:2000], ref_gb) < TOL
        ref_ga = oracle.grads(oracle.tp_simple, [a[-2000:].double(), b[-2000:].double()], go[-2000:].double())[0]
        assert relerr(ga[-2000:], ref_ga) < TOL


@pytest.mark.parametrize("n,ci,co", [(1000, 32, 64), (257, 8, 16), (33, 5, 7)])
def test_tp_weighted_forward_backward(bm, oracle, n, ci, co):
    # the 1000-atom C_in=32, C_out=64 benchmark shape first; odd channel counts exercise the tile edges
    g = torch.Generator().manual_seed(2)
    x = torch.randn(n, ci, 16, generator=g)
    v = torch.randn(n, 3, generator=g)
    Y = oracle.sh((v / v.norm(dim=1, keepdim=True)).double(), 3).float()
    W = torch.randn(34, ci, co, generator=g) / ci ** 0.5
    go = torch.randn(n, co, 16, generator=g)
    out = bm.tensor_product(x.to(dev), Y.to(dev), W.to(dev))
    assert relerr(out, oracle.tp(x.double(), Y.double(), W.double())) < TOL
    gx, gy, gw = bm.tensor_product_backward(x.to(dev), Y.to(dev), W.to(dev), go.to(dev))
    rx, ry, rw = oracle.grads(oracle.tp, [x.double(), Y.double(), W.double()], go.double())
    assert relerr(gx, rx) < TOL
    assert relerr(gy, ry) < TOL
    assert relerr(gw, rw) < TOL
    # needs_* flags skip outputs
    gx2, gy2, gw2 = bm.tensor_product_backward(x.to(dev), Y.to(dev), W.to(dev), go.to(dev), True, False, False)
    assert gy2 is None and gw2 is None and torch.equal(gx2, gx)


def test_tp_autograd_function(bm, oracle):
    g = torch.Generator().manual_seed(3)
    x = torch.randn(100, 8, 16, generator=g).to(dev).requires_grad_(True)
    Y = torch.randn(100, 16, generator=g).to(dev).requires_grad_(True)
    W = torch.randn(34, 8, 4, generator=g).to(dev).requires_grad_(True)
    out = bm.TensorProduct.apply(x, Y, W, 8, 4)
    go = torch.randn_like(out)
    gx, gy, gw = torch.autograd.grad(out, [x, Y, W], go)
    rx, ry, rw = oracle.grads(oracle.tp, [x.detach().double().cpu(), Y.detach().double().cpu(),
                                          W.detach().double().cpu()], go.double().cpu())
    assert relerr(gx, rx) < TOL and relerr(gy, ry) < TOL and relerr(gw, rw) < TOL


def test_determinism(bm):
    g = torch.Generator().manual_seed(4)
    x = torch.randn(1000, 32, 16, generator=g).to(dev)
    Y = torch.randn(1000, 16, generator=g).to(dev)
    W = torch.randn(34, 32, 64, generator=g).to(dev)
    go = torch.randn(1000, 64, 16, generator=g).to(dev)
    a = bm.tensor_product_backward(x, Y, W, go)
    b = bm.tensor_product_backward(x, Y, W, go)
    assert all(torch.equal(p, q) for p, q in zip(a, b))


def test_tp_weighted_tf32_mode(bm, oracle):
    """Single-pass TF32 channel mix: inside the 2e-3 gate of the tf32 path."""
    from batmobile._lib import lib
    g = torch.Generator().manual_seed(12)
    n, ci, co = 1000, 32, 64
    x = torch.randn(n, ci, 16, generator=g)
    Y = oracle.sh(unit(n, 13).double(), 3).float()
    W = torch.randn(34, ci, co, generator=g) / ci ** 0.5
    ref = oracle.tp(x.double(), Y.double(), W.double())
    assert lib.bm_set_mix_precision(1) == 0
    try:
        out = bm.tensor_product(x.to(dev), Y.to(dev), W.to(dev))
    finally:
        lib.bm_set_mix_precision(0)
    err = relerr(out, ref)
    assert 1e-6 < err < 2e-3
    assert relerr(bm.tensor_product(x.to(dev), Y.to(dev), W.to(dev)), ref) < TOL


def test_bounded_device_wait_times_out_cleanly(bm, oracle):
    """A device wait that can never complete gives up within its limit, reports
    BM_ERR_TIMEOUT through the error flag, and the next call runs normally."""
    import ctypes
    import time
    from batmobile._lib import lib
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.monotonic()
    assert lib.bm_selftest_wait_timeout(st) == 6   # BM_ERR_TIMEOUT
    assert time.monotonic() - t0 < 10.0
    assert lib.bm_device_error_check() == 0        # read and cleared
    v = torch.randn(1000, 3, device="cuda")
    v = v / v.norm(dim=1, keepdim=True)
    Y = bm.spherical_harmonics(v, 3)
    assert relerr(Y, oracle.sh(v.double().cpu(), 3)) < 1e-5
