"""Spatial slab decomposition of a periodic system across ranks.

The box is cut into P equal slabs along one axis.  Rank r owns the atoms whose
coordinate lies in [r L/P, (r+1) L/P) and computes every edge whose TARGET it
owns ("owner computes the incoming sum").  Sources within the cutoff of either
face live on the neighbouring ranks: each step the ranks exchange those ghost
atoms (positions, features) with their two neighbours, run the neighbour list
and the fused layer on owned + ghost atoms in global coordinates with the
global minimum image -- so the per-pair predicate, and the union of the
per-rank edge sets, equal the single-process ones bit for bit -- then send the
ghosts' gradients back to their owners (reverse halo) and sum the weight
gradient over ranks.

Communication goes through torch.distributed point-to-point batches (NCCL over
NVLink on B200s, gloo on the CPU in tests).  Per step:
  1. a header exchange with both neighbours: (magic, step id, ghost count);
     the one host read of the exchange (the counts size the receive buffers);
  2. ghost positions, then the ghost features, both posted before the host
     waits for the positions (checked on arrival); the feature transfer
     overlaps the neighbour list and the CSR build;
  3. after the backward, one batch returns the ghosts' feature and position
     gradients (reverse halo, sent as contiguous row ranges) while the
     weight-gradient all-reduce runs beside it; the compute stream waits for
     the all-reduce only after the reverse halo is posted.
Failure handling: every host-side wait polls the outstanding work against a
deadline (`timeout` seconds).  When it runs out -- a peer that died or never
sends, a truncated or mismatched message -- the process group is aborted
(NCCL) and HaloError is raised, instead of hanging every rank.  Headers that
disagree on the magic or the step id raise HaloError at once.  Device-side
waits (stream-ordered) are covered by the check at the end of the step.

The compute is pluggable (`compute.neighbors/layer/pos_grad`): GpuCompute below
calls libbatmobile_b200; tests pass a CPU implementation.  Requires a slab
width of at least cutoff + margin, so each rank only talks to its two
neighbours; with two ranks both neighbours are the same peer, and an atom near
both faces is sent once.
"""
import datetime
import time
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.distributed as dist

_MAGIC = 0x6261746D  # header tag of this exchange
_MAGIC_F = 24301.0   # trailer tag (exact in every float type)


class HaloError(RuntimeError):
    """A halo exchange or collective failed or missed its deadline."""


@dataclass
class Halo:
    """Per-step ghost bookkeeping of one rank."""
    send_left: torch.Tensor    # owned indices sent to the left neighbour
    send_right: torch.Tensor   # owned indices sent to the right neighbour
    n_from_left: int           # ghosts received from the left neighbour (its right face)
    n_from_right: int          # ghosts received from the right neighbour (its left face)


class StageEvents:
    """CUDA events at stage boundaries of a step (on the current stream);
    `ms()` gives the device time of each stage."""

    def __init__(self):
        self.names, self.events = [], []

    def mark(self, name):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.names.append(name)
        self.events.append(e)

    def ms(self):
        self.events[-1].synchronize()
        return {self.names[i]: self.events[i - 1].elapsed_time(self.events[i]) for i in range(1, len(self.events))}


class SlabDecomposition:
    def __init__(self, box, cutoff: float, world: int, rank: int, axis: int = 0, group=None,
                 margin: Optional[float] = None, timeout: Optional[float] = 120.0):
        self.box = torch.as_tensor(box, dtype=torch.float32).reshape(-1).cpu()
        if self.box.numel() == 1:
            self.box = self.box.repeat(3)
        self.L = float(self.box[axis])
        self.cutoff = float(cutoff)
        self.world, self.rank, self.axis, self.group = int(world), int(rank), int(axis), group
        self.width = self.L / self.world
        # ghosts are selected with a margin: extra ghosts only add candidates,
        # a missing one would drop edges.
        self.margin = float(margin) if margin is not None else 1e-3 * self.cutoff + 1e-4
        self.reach = self.cutoff + self.margin
        if self.world > 1 and self.width < self.reach:
            raise ValueError("slab width %.3f must be at least the cutoff + margin %.3f" % (self.width, self.reach))
        self.lo = self.rank * self.width
        self.hi = (self.rank + 1) * self.width
        self.left = (self.rank - 1) % self.world
        self.right = (self.rank + 1) % self.world
        self.timeout = timeout
        self.step_id = 0
        self._deferred = []   # (works, what) posted stream-ordered, checked at the end of the step
        self._trailers = []   # (trailer row, expected rows, what, peer) of received messages

    # ------------------------------------------------------------ ownership --
    def owner(self, pos: torch.Tensor) -> torch.Tensor:
        """Rank owning each position (coordinates wrapped into [0, L))."""
        c = pos[:, self.axis]
        c = c - torch.floor(c / self.L) * self.L
        return torch.clamp((c / self.width).floor().long(), 0, self.world - 1)

    def owned_mask(self, pos: torch.Tensor) -> torch.Tensor:
        return self.owner(pos) == self.rank

    def face_lists(self, pos_own: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Owned atoms within cutoff (+margin) of the left / right slab face.
        With two ranks both faces border the same peer: an atom near both
        faces is listed on the left only, so the peer receives it once."""
        c = pos_own[:, self.axis]
        c = c - torch.floor(c / self.L) * self.L
        near_left = c - self.lo < self.reach
        near_right = self.hi - c < self.reach
        if self.world == 2:
            near_right = near_right & ~near_left
        both = torch.stack([near_left, near_right], 0)
        nl, nr = (int(v) for v in both.sum(1).cpu().tolist())   # the one host read of the face lists
        idx = torch.nonzero_static(both, size=nl + nr)[:, 1]      # row-major: the left list, then the right
        return idx[:nl], idx[nl:]

    # ------------------------------------------------------ waits, failure --
    def abort(self):
        """Abort the communicator so that no rank stays blocked in it (NCCL)."""
        try:
            if dist.get_backend(self.group) == "nccl":
                dist.distributed_c10d._abort_process_group(self.group or dist.group.WORLD)
        except Exception:  # noqa: BLE001  (best effort: the HaloError below is what the caller sees)
            pass

    def _fail(self, what, why):
        self.abort()
        return HaloError("rank %d step %d: %s %s (neighbours %d / %d)"
                         % (self.rank, self.step_id, what, why, self.left, self.right))

    def _deadline_wait(self, works, what):
        """Block the host until every work completes, or abort and raise
        HaloError once `timeout` seconds have passed.  NCCL work is polled
        (is_completed); gloo work completes only inside wait(), which takes
        the remaining time as its own limit."""
        end = None if self.timeout is None else time.monotonic() + self.timeout
        try:
            if end is not None and dist.get_backend(self.group) == "nccl":
                spin_end = time.monotonic() + 2e-3   # poll without sleeping first (a sleep costs ~0.1 ms)
                while not all(w.is_completed() for w in works):
                    now = time.monotonic()
                    if now > end:
                        raise self._fail(what, "did not complete within %.1f s: a peer left, never sent, or sent "
                                               "a message of another size" % self.timeout)
                    if now > spin_end:
                        time.sleep(1e-4)
            for w in works:
                if end is None:
                    w.wait()
                else:
                    w.wait(timeout=datetime.timedelta(seconds=max(end - time.monotonic(), 1e-3)))
        except HaloError:
            raise
        except Exception as exc:  # noqa: BLE001  (transport error or gloo timeout)
            text = str(exc).strip().splitlines()[-1][:200] if str(exc).strip() else repr(exc)
            if "timed out" in text.lower():
                raise self._fail(what, "did not complete within %.1f s: a peer left, never sent, or sent a message "
                                       "of another size [%s]" % (self.timeout, text)) from exc
            raise self._fail(what, "failed: %s" % text) from exc

    def _stream_wait(self, works, what):
        """Order the current stream after the works without blocking the host
        (device tensors); the deadline is checked at the end of the step."""
        for w in works:
            w.wait()
        self._deferred.append((works, what))

    def _check_trailers(self):
        """Every received message ends in a trailer row (magic, step id, row
        count); a truncated or mismatched message fails here."""
        pending, self._trailers = self._trailers, []
        if not pending:
            return
        got = torch.stack([t.reshape(-1)[:3].double() for t, _, _, _ in pending]).cpu().tolist()
        for (magic, sid, n), (_, want, what, peer) in zip(got, pending):
            if magic != _MAGIC_F or sid != self.step_id or n != want:
                raise self._fail(what, "from rank %d ends in (%g, step %g, %g rows), expected (%g, step %d, %d "
                                       "rows): truncated or mismatched message"
                                 % (peer, magic, sid, n, _MAGIC_F, self.step_id, want))

    def _finish(self):
        pending, self._deferred = self._deferred, []
        for works, what in pending:
            self._deadline_wait(works, what)
        self._check_trailers()

    # ---------------------------------------------------------- exchanges --
    def _pack(self, a: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        """Rows a[idx] followed by the trailer row (magic, step id, count)."""
        n = idx.numel()
        buf = a.new_empty((n + 1,) + tuple(a.shape[1:]))
        torch.index_select(a, 0, idx, out=buf[:n])
        return self._trail(buf, n)

    def _pack_range(self, a: torch.Tensor, start: int, n: int) -> torch.Tensor:
        """Rows a[start:start + n] followed by the trailer row."""
        buf = a.new_empty((n + 1,) + tuple(a.shape[1:]))
        buf[:n].copy_(a[start:start + n])
        return self._trail(buf, n)

    def _trail(self, buf: torch.Tensor, n: int) -> torch.Tensor:
        buf[n].zero_()
        tr = buf[n].reshape(-1)
        for k, val in enumerate((_MAGIC_F, float(self.step_id), float(n))):
            tr[k].fill_(val)   # device-side fills, no host synchronisation
        return buf

    def _post(self, to_left: torch.Tensor, to_right: torch.Tensor, n_from_left: int, n_from_right: int,
              what: str):
        """Posts one exchange of packed buffers with both neighbours; returns
        (from_left, from_right, works) without the trailer rows (queued for
        the check).  Right-going traffic first (my right face -> right
        neighbour, left neighbour's right face -> me), then left-going; with
        two ranks both neighbours are the same peer and this order pairs the
        messages."""
        shape = tuple(to_left.shape[1:])
        from_left = torch.empty((n_from_left + 1,) + shape, dtype=to_left.dtype, device=to_left.device)
        from_right = torch.empty((n_from_right + 1,) + shape, dtype=to_left.dtype, device=to_left.device)
        ops = [dist.P2POp(dist.isend, to_right, self.right, self.group),
               dist.P2POp(dist.irecv, from_left, self.left, self.group),
               dist.P2POp(dist.isend, to_left, self.left, self.group),
               dist.P2POp(dist.irecv, from_right, self.right, self.group)]
        works = dist.batch_isend_irecv(ops)
        self._trailers += [(from_left[n_from_left], n_from_left, what, self.left),
                           (from_right[n_from_right], n_from_right, what, self.right)]
        return from_left[:n_from_left], from_right[:n_from_right], works

    def halo(self, pos_own: torch.Tensor) -> Halo:
        """Face lists and the header exchange (magic, step id, ghost count)."""
        left, right = self.face_lists(pos_own)
        if self.world == 1:
            return Halo(left[:0], right[:0], 0, 0)
        dev = pos_own.device
        hl = torch.tensor([[_MAGIC, self.step_id, left.numel()]], dtype=torch.int64, device=dev)
        hr = torch.tensor([[_MAGIC, self.step_id, right.numel()]], dtype=torch.int64, device=dev)
        fl = torch.empty_like(hl)
        fr = torch.empty_like(hr)
        ops = [dist.P2POp(dist.isend, hr, self.right, self.group),
               dist.P2POp(dist.irecv, fl, self.left, self.group),
               dist.P2POp(dist.isend, hl, self.left, self.group),
               dist.P2POp(dist.irecv, fr, self.right, self.group)]
        self._deadline_wait(dist.batch_isend_irecv(ops), "ghost header exchange")
        hdr = torch.cat([fl, fr], 0).cpu().tolist()
        for (magic, sid, _), peer in zip(hdr, (self.left, self.right)):
            if magic != _MAGIC or sid != self.step_id:
                raise self._fail("ghost header exchange", "from rank %d is (magic %#x, step %d): the ranks are "
                                                          "out of step" % (peer, magic, sid))
        return Halo(left, right, int(hdr[0][2]), int(hdr[1][2]))

    def post_ghosts(self, h: Halo, a: torch.Tensor, what="ghost exchange"):
        """Posts the exchange of one owned array's ghost rows; returns
        (rows from the left neighbour, rows from the right neighbour, works)."""
        return self._post(self._pack(a, h.send_left), self._pack(a, h.send_right), h.n_from_left, h.n_from_right,
                          what)

    def gather_ghosts(self, h: Halo, *owned: torch.Tensor):
        """For each owned array, the ghost rows [from_left ; from_right] (blocking)."""
        out = []
        for a in owned:
            if self.world == 1:
                out.append(a[:0])
                continue
            fl, fr, works = self.post_ghosts(h, a)
            self._deadline_wait(works, "ghost exchange")
            self._check_trailers()
            out.append(torch.cat([fl, fr], 0))
        return out

    def scatter_ghost_grads(self, h: Halo, grads_owned, grads_ghost, mark=lambda name: None):
        """Reverse halo of several arrays in one batch: each ghost gradient goes
        back to its owner and is added to the owner's row (fixed order: the
        returns from the left neighbour, then the right's).  Returns the
        summed owned gradients.  `mark` records stage boundaries (packing,
        transfer, sum)."""
        if self.world == 1:
            return list(grads_owned)
        ops, rets = [], []
        for gown, gg in zip(grads_owned, grads_ghost):
            nl, nr = h.n_from_left, h.n_from_right
            gl = self._pack_range(gg, 0, nl)
            gr = self._pack_range(gg, nl, nr)
            shape = tuple(gg.shape[1:])
            ns_l, ns_r = h.send_left.numel(), h.send_right.numel()
            ret_right = torch.empty((ns_r + 1,) + shape, dtype=gg.dtype, device=gg.device)
            ret_left = torch.empty((ns_l + 1,) + shape, dtype=gg.dtype, device=gg.device)
            ops += [dist.P2POp(dist.isend, gl, self.left, self.group),
                    dist.P2POp(dist.irecv, ret_right, self.right, self.group),
                    dist.P2POp(dist.isend, gr, self.right, self.group),
                    dist.P2POp(dist.irecv, ret_left, self.left, self.group)]
            self._trailers += [(ret_right[ns_r], ns_r, "reverse halo", self.right),
                               (ret_left[ns_l], ns_l, "reverse halo", self.left)]
            rets.append((ret_left[:ns_l], ret_right[:ns_r]))
        mark("reverse_pack")
        works = dist.batch_isend_irecv(ops)
        if grads_owned[0].is_cuda:
            self._stream_wait(works, "reverse halo")
        else:
            self._deadline_wait(works, "reverse halo")
        mark("reverse_transfer")
        out = []
        for gown, (ret_left, ret_right) in zip(grads_owned, rets):
            gown.index_add_(0, h.send_left, ret_left)    # in place: the owned rows of the step's own gradient
            gown.index_add_(0, h.send_right, ret_right)
            out.append(gown)
        return out

    def allreduce_sum(self, t: torch.Tensor, block: bool = True):
        """Sums t over the ranks in place.  block=False on device tensors posts
        the all-reduce and returns (t, works) for `_stream_wait` later, so
        that the current stream is not held behind it meanwhile."""
        if self.world > 1:
            w = dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
            if block or not t.is_cuda:
                self._deadline_wait([w], "weight-gradient all-reduce")
            else:
                return t, [w]
        return t if block or not t.is_cuda else (t, [])

    # ---------------------------------------------------------------- step --
    def step(self, compute, pos_own, x_own, W, G_own, stages: Optional[StageEvents] = None):
        """One sharded layer step: halo exchange, local neighbour list over
        owned rows, fused layer forward and backward, reverse halo, dW sum.
        Returns (out_own, grad_x_own, grad_W, grad_pos_own, local_edges).
        `stages` (optional) records a CUDA event after each stage."""
        mark = stages.mark if stages is not None else (lambda name: None)
        self.step_id += 1
        self._deferred, self._trailers = [], []
        n_own = pos_own.shape[0]
        mark("start")
        h = self.halo(pos_own)
        self.last_halo = h
        mark("halo_header")
        if self.world > 1:
            pl, pr, wp = self.post_ghosts(h, pos_own, "ghost position exchange")
            pos_trailers, self._trailers = self._trailers, []
            xl, xr, wx = self.post_ghosts(h, x_own, "ghost feature exchange")  # overlaps the neighbour list
            self._deadline_wait(wp, "ghost position exchange")
            feat_trailers, self._trailers = self._trailers, pos_trailers
            self._check_trailers()   # the neighbour list must not see a truncated position message
            self._trailers = feat_trailers
            pos_l = torch.cat([pos_own, pl, pr], 0)
        else:
            pos_l = pos_own
        mark("halo_positions")
        src, dst, vec, graph = compute.neighbors(pos_l, n_own, self.box, self.cutoff)
        mark("neighbor_list")
        if self.world > 1:
            if x_own.is_cuda:
                self._stream_wait(wx, "ghost feature exchange")
            else:
                self._deadline_wait(wx, "ghost feature exchange")
            x_l = torch.cat([x_own, xl, xr], 0)
        else:
            x_l = x_own
        mark("halo_features")
        # the upstream gradient exists for the owned rows only (ghost rows are not targets)
        out_l, gx_l, gv, gW = compute.layer(x_l, vec, W, src, dst, graph, G_own, mark)
        gpos_l = compute.pos_grad(gv, src, dst, graph, pos_l.shape[0])
        mark("pos_grad")
        gW = self.allreduce_sum(gW, block=False)
        if isinstance(gW, tuple):   # device tensors: the stream waits for it after the reverse halo is posted
            gW, w_ar = gW
        else:
            w_ar = []
        gx_own, gpos_own = self.scatter_ghost_grads(h, [gx_l[:n_own], gpos_l[:n_own]],
                                                    [gx_l[n_own:], gpos_l[n_own:]], mark)
        if w_ar:
            self._stream_wait(w_ar, "weight-gradient all-reduce")
        mark("reverse_sum_allreduce")
        self._finish()
        return out_l[:n_own], gx_own, gW, gpos_own, int(src.numel())


class GpuCompute:
    """Local compute on libbatmobile_b200: the row-restricted neighbour list gives
    each owned atom's incoming edges already grouped by target."""

    def neighbors(self, pos_l, n_rows, box, cutoff):
        from . import _batmobile as _bm
        ei, vec, rp = _bm.neighbor_list(pos_l.contiguous(), box, cutoff, return_row_ptr=True, n_rows=n_rows)
        # row j (owned) lists neighbours i: the message edge is i -> j with vector p_j - p_i
        dst, src = ei[0].contiguous(), ei[1].contiguous()
        e = src.numel()
        ident = torch.arange(e, dtype=torch.int64, device=src.device)
        flipped = torch.stack([dst, src], 0).contiguous()
        rps, ps = _bm.edge_index_to_csr(flipped, pos_l.shape[0])  # grouped by source
        graph = (rp, ident, rps, ps, int(n_rows))
        return src, dst, (-vec).contiguous(), graph

    def layer(self, x_l, vec, W, src, dst, graph, G_own, mark=lambda name: None):
        """Owned atoms (the first n_rows) are the only targets: the forward, the
        slot gradients and the weight gradient skip the ghost rows; ghosts stay
        sources, so grad_x covers every local atom.  G_own: upstream gradient of
        the owned rows.  Returns out for the owned rows."""
        from . import _batmobile as _bm
        rp, ident, rps, ps, n_own = graph
        rpt = rp[:n_own + 1]
        out, slots = _bm.layer_forward(x_l.contiguous(), vec, W, src, rpt, ident, n_targets=n_own)
        mark("layer_fwd")
        gx, gv, gw = _bm.layer_backward(x_l.contiguous(), vec, W, src, dst, rpt, ident, rps, ps, slots,
                                        G_own.contiguous(), n_targets=n_own)
        mark("layer_bwd")
        return out, gx, gv, gw

    def pos_grad(self, gv, src, dst, graph, n_local):
        from . import _batmobile as _bm
        rp, ident, rps, ps, _ = graph
        return _bm.edge_grad_to_pos(gv, rp, ident, rps, ps)
