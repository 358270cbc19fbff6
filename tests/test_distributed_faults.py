"""Failure handling of the slab decomposition, on CPU ranks (gloo): faults are
made on the host -- a truncated ghost message, a ghost count that disagrees
with the data, a rank that never sends, a rank that leaves between steps,
ranks out of step -- and every surviving rank must raise HaloError within its
deadline instead of hanging.  Also the two-rank case with a slab narrower than
twice the cutoff, where an atom near both faces must reach the peer once."""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT, PKG, relerr

DEADLINE = 3.0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _system(n, box, c, seed=11):
    g = torch.Generator().manual_seed(seed)
    pos = torch.rand(n, 3, generator=g) * box
    x = torch.randn(n, c, 16, generator=g, dtype=torch.float64)
    W = torch.randn(34, c, c, generator=g, dtype=torch.float64)
    G = torch.randn(n, c, 16, generator=g, dtype=torch.float64)
    return pos, x, W, G


def _put_and_exit(q, item):
    q.put(item)
    q.close()
    q.join_thread()   # flush the queue before leaving without teardown
    os._exit(0)


def _worker(rank, world, port, q, fault, n, box, rc, c):
    import sys
    for pth in (ROOT, PKG, os.path.join(ROOT, "tests")):
        if pth not in sys.path:
            sys.path.insert(0, pth)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from batmobile.distributed import SlabDecomposition, HaloError
    from test_distributed_cpu import CpuCompute

    class Faulty(SlabDecomposition):
        def _pack(self, a, idx):
            if fault == "truncated" and self.step_id == 2 and self.rank == 1 and a.dtype == torch.float64:
                idx = idx[:-1]   # the feature message loses a row; the header promised all of them
            return super()._pack(a, idx)

        def halo(self, pos_own):
            h = super().halo(pos_own)
            if fault == "count" and self.step_id == 2 and self.rank == 0:
                h.n_from_left += 1   # this rank expects one ghost more than the peer sends
            return h

    pos, x, W, G = _system(n, box, c)
    sd = Faulty([box] * 3, rc, world, rank, timeout=DEADLINE)
    own = torch.nonzero(sd.owned_mask(pos)).flatten()
    args = (CpuCompute(), pos[own], x[own], W, G[own])
    status, msg, t = "ok", "", 0.0
    try:
        sd.step(*args)                       # step 1 is clean in every mode
        if fault == "leave" and rank == 1:
            _put_and_exit(q, (rank, "left", "", 0.0))
        if fault == "never" and rank == 1:
            time.sleep(3 * DEADLINE)         # alive, but never joins step 2
            _put_and_exit(q, (rank, "slept", "", 0.0))
        if fault == "out_of_step" and rank == 1:
            sd.step_id += 1
        t0 = time.monotonic()
        try:
            r = sd.step(*args)
            status = "ok"
            if fault == "none":
                msg = r
        except HaloError as e:
            status, msg = "halo_error", str(e)
        t = time.monotonic() - t0
    except Exception as e:  # noqa: BLE001
        status, msg = "other_error", repr(e)
    if fault == "none" and status == "ok":
        out, gx, gw, gp, e = msg
        arrays = tuple(a.detach().numpy() for a in (out, gx, gw, gp, own))   # by value: no shared-memory handles
        _put_and_exit(q, (rank, status, arrays + (e,), t))
    _put_and_exit(q, (rank, status, msg, t))   # no collective teardown after a fault


def _run(fault, world=2, n=400, box=16.0, rc=3.0, c=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fault, n, box, rc, c)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=120)
        res[r[0]] = r[1:]
    for p in procs:
        p.join(timeout=30)
    return res


@pytest.mark.parametrize("fault,expect", [
    ("truncated", "truncated or mismatched"),
    ("count", ""),
    ("never", "did not complete"),
    ("leave", ""),
    ("out_of_step", "out of step"),
])
def test_fault_raises_halo_error_within_deadline(fault, expect):
    res = _run(fault)
    status, msg, t = res[0]
    assert status == "halo_error", (fault, res)
    assert expect in msg, msg
    assert t < DEADLINE + 5.0, (fault, t)


def _reference(n, box, rc, c):
    from oracle import ref_ops
    pos, x, W, G = _system(n, box, c)
    ei, vec = ref_ops.nl_cells(pos, [box] * 3, rc)
    p = pos.double().clone().requires_grad_(True)
    ins = [x.clone().requires_grad_(True), W.clone().requires_grad_(True)]
    d = p[ei[1]] - p[ei[0]]
    v = d - torch.round(d / box) * box
    out = ref_ops.interaction(ins[0], v, ins[1], ei, n)
    gx, gw, gp = torch.autograd.grad(out, [ins[0], ins[1], p], G)
    return out.detach(), gx, gw, gp, ei.shape[1]


def test_two_ranks_narrow_slabs_send_each_ghost_once():
    """Slab width 5 between rc = 3 and 2 rc: atoms within reach of both faces
    exist; the sharded step must still equal the single-process one."""
    n, box, rc, c = 300, 10.0, 3.0, 2
    res = _run("none", world=2, n=n, box=box, rc=rc, c=c)
    ref_out, ref_gx, ref_gw, ref_gp, E = _reference(n, box, rc, c)
    tot = 0
    for rank in (0, 1):
        status, payload, _ = res[rank]
        assert status == "ok", res[rank]
        out, gx, gw, gp, own, e = payload
        out, gx, gw, gp, own = (torch.from_numpy(a) for a in (out, gx, gw, gp, own))
        assert relerr(out, ref_out[own]) < 1e-6 and relerr(gx, ref_gx[own]) < 1e-6
        assert relerr(gp, ref_gp[own]) < 1e-6 and relerr(gw, ref_gw) < 1e-6
        tot += e
    assert tot == E


def test_slab_narrower_than_reach_rejected():
    import sys
    sys.path.insert(0, PKG)
    from batmobile.distributed import SlabDecomposition
    with pytest.raises(ValueError):
        SlabDecomposition([10.0] * 3, 5.0, 2, 0)
    SlabDecomposition([10.2] * 3, 5.0, 2, 0)
