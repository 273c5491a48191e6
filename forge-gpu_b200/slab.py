"""x-slab domain decomposition of the SPH step across ranks (one process per GPU).

The reference has no multi-GPU path (its P2P API is stubbed, forge-runtime/src/
cuda.rs:134-178); this is the sharded form of the manifest SPH step for large
runs. Rank r owns the particles with x in [lo_r, hi_r) (rank 0 also owns
x < lo_0, the last rank x >= hi). Every step:

  1. halo: owned particles within h of a slab face are sent to that neighbour
     (pos, vel, id) and appended there as ghosts;
  2. grid + density over owned + ghosts (the global grid geometry on every
     rank, so cells, windows and pair sets are those of the single-device run);
  3. ghost-density exchange: each owner sends the exact densities of the
     particles it sent, which overwrite the ghosts' partial ones;
  4. force + gravity/integrate/box for the owned particles only;
  5. migration: owned particles that left the slab move to the neighbour.

Only the two neighbour exchanges cross ranks (send/recv of counts, then
payloads), no data-path collective; on GPU ranks (comm="nccl") steps 3 and
5 run beside the interior half of step 4 (SlabRun._step_overlapped). Skewed
inputs move the slab bounds every k steps (SlabRun.rebalance: one
all-reduce of a work histogram). The per-rank compute is a Backend:
GpuBackend runs the library's kernels (forge_sph_density,
forge_sph_force_step[_zone]) on the rank's GPU; tests supply a CPU backend
and, for failure detection, an in-process transport (MailboxHub).
With ``order_by_id`` local arrays are kept in particle-id order, which makes
each particle's neighbour order, and hence the result, identical to the
single-device run.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

# Payload columns: x, y, z, vx, vy, vz, id (int32 bits carried in a float32).
_NCOL = 7


class SlabGeometry:
    """x-slabs of [x0, x1): uniform, or at explicit bounds b_0 < ... < b_W."""

    def __init__(self, rank: int, world: int, x0: float, x1: float, h: float, bounds=None):
        self.rank, self.world, self.h = rank, world, h
        if bounds is None:
            w = (x1 - x0) / world
            bounds = [x0 + w * k for k in range(world)] + [x1]
        self.set_bounds(bounds)
        self.first = rank == 0
        self.last = rank == world - 1

    def set_bounds(self, bounds) -> None:
        self.bounds = [float(b) for b in bounds]
        self.lo = self.bounds[self.rank]
        self.hi = self.bounds[self.rank + 1]

    def force_zones(self, reach: float, margin: float | None = None):
        """(inner_lo, inner_hi, guard_lo, guard_hi) in float32 for the split
        force pass. An interior particle must start and end the step at
        least `reach` inside every face that has a neighbour (guard), so no
        halo or migrant list can see it; the interior zone starts `margin`
        (default h/4, the largest displacement allowed in one step) further
        in. Sums in float32, like the classification's lo + reach."""
        f32 = np.float32
        inf = f32(np.inf)
        lo, hi, r = f32(self.lo), f32(self.hi), f32(reach)
        m = f32(self.h / 4 if margin is None else margin)
        if self.first:
            inner_lo = guard_lo = -inf
        else:
            guard_lo = lo + r
            inner_lo = guard_lo + m
        if self.last:
            inner_hi = guard_hi = inf
        else:
            guard_hi = hi - r
            inner_hi = guard_hi - m
        return float(inner_lo), float(inner_hi), float(guard_lo), float(guard_hi)

    def owned_mask(self, x: torch.Tensor) -> torch.Tensor:
        m = torch.ones_like(x, dtype=torch.bool)
        if not self.first:
            m &= x >= self.lo
        if not self.last:
            m &= x < self.hi
        return m


def quantile_bounds(hist, x0: float, x1: float, world: int):
    """Bounds b_0 = x0 < ... < b_W = x1 at the particle-count quantiles of
    an x-histogram (bins over [x0, x1), linear inside a bin)."""
    hist = np.asarray(hist, dtype=np.float64)
    nb = hist.size
    edges = x0 + (x1 - x0) * np.arange(nb + 1) / nb
    cum = np.concatenate([[0.0], np.cumsum(hist)])
    total = cum[-1]
    if total <= 0:
        return [x0 + (x1 - x0) * k / world for k in range(world)] + [x1]
    out = [float(x0)]
    for k in range(1, world):
        q = total * k / world
        j = min(max(int(np.searchsorted(cum, q, side="right")) - 1, 0), nb - 1)  # bin holding the quantile
        frac = (q - cum[j]) / hist[j] if hist[j] > 0 else 0.0
        out.append(float(edges[j] + frac * (edges[j + 1] - edges[j])))
    out.append(float(x1))
    return out


def min_width_bounds(b, min_width: float):
    """b with every slab at least min_width wide (inner bounds pushed right,
    then left), rounded to float32 (the library compares in float32)."""
    b = list(b)
    for k in range(1, len(b) - 1):
        b[k] = max(b[k], b[k - 1] + min_width)
    for k in range(len(b) - 2, 0, -1):
        b[k] = min(b[k], b[k + 1] - min_width)
    return [float(np.float32(v)) for v in b]


def balanced_bounds(hist, x0: float, x1: float, old, min_width: float):
    """Rebalanced slab bounds: the quantile bounds of a global x-histogram,
    each inner bound kept between the old bounds of its neighbours (so no
    particle moves more than one slab) and every slab at least min_width
    wide (so halos come from direct neighbours only). Returns the old bounds
    when no such move exists. Pure host arithmetic on identical inputs:
    every rank computes the same bounds."""
    w = len(old) - 1
    q = quantile_bounds(hist, x0, x1, w)
    new = [float(old[0])] + [min(max(q[k], old[k - 1]), old[k + 1]) for k in range(1, w)] + [float(old[w])]
    new = min_width_bounds(new, min_width)
    ok = all(new[k + 1] - new[k] >= min_width * (1 - 1e-6) for k in range(w)) and all(
        old[k - 1] <= new[k] <= old[k + 1] for k in range(1, w))
    return new if ok else list(old)


class Exchanger:
    """Neighbour send/recv of variable-length row blocks over torch.distributed.
    With NCCL the blocks go device to device (NVLink); comm_device="cpu"
    stages them through host memory for backends that only move host
    tensors (gloo)."""

    def __init__(self, dist, rank: int, world: int, device: torch.device, comm_device=None):
        self.dist, self.rank, self.world = dist, rank, world
        self.device = torch.device(comm_device) if comm_device is not None else device
        self.home = device

    def _p2p(self, sends: dict, recvs: dict) -> None:
        if hasattr(self.dist, "exchange"):  # an in-process transport (MailboxHub)
            self.dist.exchange(sends, recvs)
            return
        ops = []
        for peer, t in sends.items():
            ops.append(self.dist.P2POp(self.dist.isend, t, peer))
        for peer, t in recvs.items():
            ops.append(self.dist.P2POp(self.dist.irecv, t, peer))
        if ops:
            for r in self.dist.batch_isend_irecv(ops):
                r.wait()

    def swap_counted(self, to_left, counts_left, to_right, counts_right, ncol: int):
        """swap() that also carries a tuple of sub-block sizes per message.
        Returns (from_left, from_right, counts_from_left, counts_from_right)."""
        left = self.rank - 1 if self.rank > 0 else None
        right = self.rank + 1 if self.rank < self.world - 1 else None
        k = len(counts_left)
        sends, recvs, cnt = {}, {}, {}
        for peer, c in ((left, counts_left), (right, counts_right)):
            if peer is None:
                continue
            sends[peer] = torch.tensor(list(c), dtype=torch.int64, device=self.device)
            cnt[peer] = torch.zeros(k, dtype=torch.int64, device=self.device)
            recvs[peer] = cnt[peer]
        self._p2p(sends, recvs)
        host = {p: tuple(int(v) for v in t.tolist()) for p, t in cnt.items()}
        zero = tuple([0] * k)
        cl, cr = host.get(left, zero), host.get(right, zero)
        a, b = self.swap_known(to_left, sum(cl), to_right, sum(cr), ncol)
        return a, b, cl, cr

    def swap_known(self, to_left, n_from_left: int, to_right, n_from_right: int, ncol: int):
        """Exchange row blocks whose incoming sizes are already known."""
        left = self.rank - 1 if self.rank > 0 else None
        right = self.rank + 1 if self.rank < self.world - 1 else None
        sends, recvs, out = {}, {}, {}
        for peer, blk, k in ((left, to_left, n_from_left), (right, to_right, n_from_right)):
            if peer is None:
                continue
            out[peer] = torch.empty((k, ncol), dtype=torch.float32, device=self.device)
            if k:
                recvs[peer] = out[peer]
            if blk.shape[0]:
                sends[peer] = blk.to(self.device).contiguous()
        self._p2p(sends, recvs)
        empty = torch.empty((0, ncol), dtype=torch.float32, device=self.home)
        a = out[left].to(self.home) if left is not None else empty
        b = out[right].to(self.home) if right is not None else empty
        return a, b


class ExchangeTimeout(RuntimeError):
    """A neighbour's message did not arrive in time (a failed or stalled
    rank); raised by the rank that waited."""


class MailboxHub:
    """In-process transport for ranks run as threads: the send/recv and
    all-reduce subset of torch.distributed that the slab exchange uses, with
    injected faults for failure-detection tests.

    delay = (lo, hi) seconds of random sleep before each send; drop(src, dst,
    seq) -> True discards that message (seq counts messages per src -> dst
    pair); a receive that waits longer than `timeout` raises ExchangeTimeout.
    Messages between a pair are FIFO, as NCCL's and gloo's are."""

    def __init__(self, world: int, timeout: float = 10.0, delay=(0.0, 0.0), drop=None, seed: int = 0):
        import queue
        import random
        import threading
        self.world, self.timeout, self.delay, self.drop = world, timeout, delay, drop
        self._q = {(a, b): queue.Queue() for a in range(world) for b in range(world)}
        self._seq = {k: 0 for k in self._q}
        self._rng = random.Random(seed)
        self._lock = threading.Lock()
        self._barrier = threading.Barrier(world, timeout=timeout)
        self._acc = None

    def rank(self, r: int) -> "MailboxRank":
        return MailboxRank(self, r)


class MailboxRank:
    """One rank's view of a MailboxHub (passed where torch.distributed is)."""

    def __init__(self, hub: MailboxHub, rank: int):
        self.hub, self.r = hub, rank

    def get_backend(self) -> str:
        return "mailbox"

    def get_rank(self) -> int:
        return self.r

    def exchange(self, sends: dict, recvs: dict) -> None:
        import queue
        import time
        h = self.hub
        for peer, t in sends.items():
            with h._lock:
                seq = h._seq[(self.r, peer)]
                h._seq[(self.r, peer)] += 1
                pause = h._rng.uniform(*h.delay)
            if pause:
                time.sleep(pause)
            if h.drop is not None and h.drop(self.r, peer, seq):
                continue
            h._q[(self.r, peer)].put(t.detach().clone())
        for peer, out in recvs.items():
            try:
                msg = h._q[(peer, self.r)].get(timeout=h.timeout)
            except queue.Empty:
                raise ExchangeTimeout(f"rank {self.r}: no message from rank {peer} within {h.timeout} s") from None
            if msg.shape != out.shape:
                raise ExchangeTimeout(f"rank {self.r}: message from rank {peer} has shape {tuple(msg.shape)}, "
                                      f"expected {tuple(out.shape)} (a lost message shifted the stream)")
            out.copy_(msg)

    def all_reduce(self, t: torch.Tensor) -> None:
        import threading
        h = self.hub
        try:
            with h._lock:
                h._acc = t.detach().clone() if h._acc is None else h._acc + t
            h._barrier.wait()
            t.copy_(h._acc)
            if h._barrier.wait() == 0:
                h._acc = None
            h._barrier.wait()
        except threading.BrokenBarrierError:
            raise ExchangeTimeout(f"rank {self.r}: all-reduce partner missing after {h.timeout} s") from None

    def broadcast_object_list(self, objs, src=0):
        raise NotImplementedError("the library's NCCL exchange needs real ranks")


class PyComm:
    """The two exchange rounds in Python over torch.distributed (any backend;
    gloo for CPU ranks and tests). Same protocol as the library's NCCL path."""

    def __init__(self, run, dist, comm_device=None):
        self.run = run
        self.ex = Exchanger(dist, run.geo.rank, run.geo.world, run.device, comm_device)

    def exchange(self, migrate: bool) -> None:
        """Round 1: migrants leave, [migrants | halo] go to each neighbour,
        arrivals and ghosts are appended."""
        run = self.run
        g, C, be = run.geo, run.cols, run.backend
        n_own = run.n
        flags = (0 if g.first else 1) | (0 if g.last else 2)
        if migrate:
            mig, mig_l, mig_r = be.classify(C[0], n_own, g.lo, g.hi, run.reach, flags)
        else:
            mig = mig_l = mig_r = torch.empty(0, dtype=torch.int64, device=C.device)
        rows_ml, rows_mr = C[:, mig_l], C[:, mig_r]  # gathered before the compaction moves columns
        be.compact(C, n_own, mig)
        keep = n_own - mig.numel()
        _, hl, hr = be.classify(C[0], keep, g.lo, g.hi, run.reach, flags | 4)
        send_l = torch.cat([rows_ml, C[:, hl]], dim=1).t()
        send_r = torch.cat([rows_mr, C[:, hr]], dim=1).t()
        got_l, got_r, cnt_l, cnt_r = self.ex.swap_counted(send_l, (mig_l.numel(), hl.numel()),
                                                          send_r, (mig_r.numel(), hr.numel()), _NCOL)
        am_l, ah_l = cnt_l
        am_r, ah_r = cnt_r
        n_new = keep + am_l + am_r
        ng = ah_l + ah_r + mig_l.numel() + mig_r.numel()
        run._need(n_new + ng + 1)
        C[:, keep:keep + am_l] = got_l[:am_l].t()
        C[:, keep + am_l:n_new] = got_r[:am_r].t()
        o = n_new
        blocks = {}
        for name, blk in (("hl", got_l[am_l:].t()), ("hr", got_r[am_r:].t()), ("ml", rows_ml), ("mr", rows_mr)):
            w = blk.shape[1]
            C[:, o:o + w] = blk
            blocks[name] = torch.arange(o, o + w, device=C.device)
            o += w
        arr_l = torch.arange(keep, keep + am_l, device=C.device)
        arr_r = torch.arange(keep + am_l, n_new, device=C.device)
        # round 2: rho of [halo sent to X, arrivals from X] goes to X; X's rho
        # fills [halo from X, our migrants to X] in the same order.
        self.rho_send = (torch.cat([hl, arr_l]), torch.cat([hr, arr_r]))
        self.rho_slot = (torch.cat([blocks["hl"], blocks["ml"]]), torch.cat([blocks["hr"], blocks["mr"]]))
        run.n, run.ng = n_new, ng

    def set_bounds(self, lo: float, hi: float) -> None:
        pass  # reads run.geo

    def exchange_rho(self, rho: torch.Tensor) -> None:
        """Round 2: ghosts receive their owners' densities."""
        send_l, send_r = self.rho_send
        slot_l, slot_r = self.rho_slot
        got_l, got_r = self.ex.swap_known(rho[send_l].reshape(-1, 1), slot_l.numel(),
                                          rho[send_r].reshape(-1, 1), slot_r.numel(), 1)
        rho[slot_l] = got_l.flatten()
        rho[slot_r] = got_r.flatten()


class NcclComm:
    """The two exchange rounds inside libforge_sph (forge_slab_exchange,
    forge_slab_exchange_rho) over the library's own NCCL communicator: no
    Python between the kernels and the NCCL calls of a round."""

    def __init__(self, run, dist, forge_sph):
        self.run, self.f = run, forge_sph
        self.L = forge_sph.lib()
        uid = ctypes.create_string_buffer(128)
        if run.geo.rank == 0:
            forge_sph.check(self.L.forge_nccl_unique_id(uid))
        obj = [uid.raw if run.geo.rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = ctypes.create_string_buffer(obj[0], 128)
        h = ctypes.c_void_p()
        forge_sph.check(self.L.forge_slab_comm_create(uid, run.geo.rank, run.geo.world, run.device.index,
                                                      run.capacity, run.geo.lo, run.geo.hi, run.reach,
                                                      ctypes.byref(h)))
        self.h = h

    def __del__(self):
        h = getattr(self, "h", None)
        if h and self.f._lib is not None:
            self.f._lib.forge_slab_comm_destroy(h)
            self.h = None

    def exchange(self, migrate: bool) -> None:
        run = self.run
        n_own, ng = ctypes.c_uint64(), ctypes.c_uint64()
        self.f.check(self.L.forge_slab_exchange(self.h, run.cols.data_ptr(), run.cols.stride(0), run.n,
                                                1 if migrate else 0, ctypes.byref(n_own), ctypes.byref(ng),
                                                torch.cuda.current_stream().cuda_stream))
        run.n, run.ng = n_own.value, ng.value

    split = True  # supports the exchange overlapped with the interior force pass

    def set_bounds(self, lo: float, hi: float) -> None:
        self.f.check(self.L.forge_slab_comm_set_bounds(self.h, lo, hi))

    def exchange_begin(self) -> None:
        run = self.run
        self.f.check(self.L.forge_slab_exchange_begin(self.h, run.cols.data_ptr(), run.cols.stride(0), run.n,
                                                      torch.cuda.current_stream().cuda_stream))

    def exchange_end(self) -> None:
        run = self.run
        n_own, ng = ctypes.c_uint64(), ctypes.c_uint64()
        self.f.check(self.L.forge_slab_exchange_end(self.h, run.cols.data_ptr(), run.cols.stride(0),
                                                    ctypes.byref(n_own), ctypes.byref(ng),
                                                    torch.cuda.current_stream().cuda_stream))
        run.n, run.ng = n_own.value, ng.value

    def exchange_rho(self, rho: torch.Tensor) -> None:
        self.f.check(self.L.forge_slab_exchange_rho(self.h, rho.data_ptr(), torch.cuda.current_stream().cuda_stream))


class SlabRun:
    """One rank's share of a sharded SPH run.

    Particle state lives in one preallocated (7, capacity) float32 buffer,
    rows x, y, z, vx, vy, vz, id-bits, so each row slice cols[k, :n] is a
    contiguous SoA array the kernels take directly: owned particles in
    columns [0, n), ghosts (copies of neighbours' particles within h of a
    face) after them.

    Two neighbour exchange rounds per step:
      round 1 (after force, for the next step): migrants (owned particles that
        left the slab) and halo rows (owned particles within h of a face) go
        to that neighbour in one message; the receiver appends migrants to its
        owned set and halo rows as ghosts. The sender keeps its migrants as
        ghosts too -- they sit just across the face.
      round 2 (after density): for every ghost the owner sends its exact
        density (counts known from round 1, so no count exchange).
    Leaving particles are removed by moving tail columns into their holes, so
    per step only halo- and migrant-sized data moves. comm="nccl" runs both
    rounds in the library (GPU ranks, NCCL); comm="torch" runs them in Python
    over torch.distributed (gloo / CPU ranks).
    """

    def __init__(self, dist, rank: int, world: int, cfg, pos, vel, backend, device: torch.device,
                 x_range=(0.0, 1.0), order_by_id: bool = False, comm_device=None, capacity: int | None = None,
                 comm: str = "torch", forge_sph=None, balance: bool = False, hist_bins: int = 4096,
                 halo_width: float = 1.0):
        self.cfg, self.backend, self.device = cfg, backend, device
        self.dist, self.x_range, self.hist_bins = dist, x_range, hist_bins
        # halo_width 2: ghosts within 2h of a face, so the ghosts within h get
        # their exact densities locally and round 2 (ghost densities) is skipped
        if halo_width not in (1.0, 2.0):
            raise ValueError("halo_width is 1 (h, ghost densities exchanged) or 2 (2h, computed locally)")
        self.reach = cfg.h * halo_width * (1.0 + 1e-5)
        self.local_ghost_density = halo_width == 2.0
        self.geo = SlabGeometry(rank, world, x_range[0], x_range[1], cfg.h)
        if balance:  # initial bounds at the quantiles of the (identical on every rank) initial positions
            hist = np.histogram(np.asarray(pos[0], np.float64), bins=hist_bins, range=x_range)[0]
            self.geo.set_bounds(min_width_bounds(quantile_bounds(hist, x_range[0], x_range[1], world),
                                                 2.0 * self.reach))
        self.order_by_id = order_by_id
        px = torch.as_tensor(pos[0])
        m = self.geo.owned_mask(px)
        ids = torch.arange(px.numel(), dtype=torch.int32)[m]
        own = torch.stack([torch.as_tensor(a)[m] for a in list(pos) + list(vel)] + [ids.view(torch.float32)])
        n_own = own.shape[1]
        cap = capacity if capacity is not None else int(n_own * 1.5) + 4096
        self.cols = torch.empty((_NCOL, cap), dtype=torch.float32, device=device)
        self.cols[:, :n_own] = own.to(device)
        self.n = n_own
        self.ng = 0
        self.timing = None  # set to a list to record per-phase CUDA events
        self.timing_side = []
        self._hp = None  # high-priority stream of the split force pass
        self.balance = balance
        self._work_hist = None  # x-histogram of the last step's pair work (balancing runs)
        self.comm = NcclComm(self, dist, forge_sph) if comm == "nccl" else PyComm(self, dist, comm_device)
        self.comm.exchange(migrate=False)  # initial halo

    def _x_hist(self, x: torch.Tensor, w: torch.Tensor | None) -> torch.Tensor:
        lo, hi = self.x_range
        nb = self.hist_bins
        idx = ((x.double() - lo) * (nb / (hi - lo))).floor().clamp_(0, nb - 1).long()
        return torch.bincount(idx, weights=None if w is None else w.double(), minlength=nb).double()

    def _note_work(self, x: torch.Tensor, rho: torch.Tensor) -> None:
        """Work histogram of the owned particles at density time (balancing
        runs only): each particle weighs its density, which is proportional
        to its neighbour count and so to its share of the pair work."""
        if self.balance:
            self._work_hist = self._x_hist(x, rho)

    def rebalance(self) -> bool:
        """Moves the slab bounds to the quantiles of a global x-histogram (one
        all-reduce of hist_bins values, the only collective of the sharded
        path), then reruns round 1 so particles outside the new slab migrate
        and the halos match. The histogram is the work histogram of the last
        step (skewed inputs balance pair work, not particle counts), or the
        owned particles' counts before any step. Between steps only. Returns
        whether the bounds moved."""
        hist = self._work_hist if self._work_hist is not None else self._x_hist(self.cols[0, :self.n], None)
        if self.device.type == "cuda" and self.dist.get_backend() != "nccl":
            hist = hist.cpu()
        self.dist.all_reduce(hist)
        lo, hi = self.x_range
        new = balanced_bounds(hist.cpu().numpy(), lo, hi, self.geo.bounds, 2.0 * self.reach)
        if new == self.geo.bounds:
            return False
        self.geo.set_bounds(new)
        self.comm.set_bounds(self.geo.lo, self.geo.hi)
        self.ng = 0  # ghosts of the old bounds
        self._work_hist = None
        self.comm.exchange(migrate=True)
        return True

    def _mark(self, name):
        if self.timing is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.timing.append((name, ev))

    def _mark_side(self, name):
        """Event on the current (side) stream, timed from the step's
        "prepare" mark on the main stream (the overlapped rounds' progress)."""
        if self.timing is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            ref = next(e for k, e in reversed(self.timing) if k == "prepare")
            self.timing_side.append((name, ev, ref))

    @property
    def capacity(self) -> int:
        return self.cols.shape[1]

    @property
    def n_own(self) -> int:
        return self.n

    @property
    def last_halo(self) -> int:
        return self.ng

    @property
    def state(self) -> torch.Tensor:
        """(n_own, 7) view: x, y, z, vx, vy, vz, id bits."""
        return self.cols[:, :self.n].t()

    def ids(self) -> torch.Tensor:
        return self.cols[6, :self.n].view(torch.int32)

    def _need(self, n: int) -> None:
        if n > self.capacity:
            raise RuntimeError(f"slab rank {self.geo.rank}: {n} particles exceed capacity {self.capacity}")

    def step(self) -> None:
        if getattr(self.comm, "split", False) and not self.order_by_id:
            self._step_overlapped()
            return
        C = self.cols
        self._mark("start")
        n_own, n = self.n, self.n + self.ng
        perm = None
        if self.order_by_id:  # test mode: neighbour order identical to the unsharded run
            perm = torch.argsort(C[6, :n].view(torch.int32), stable=True)
            C[:, :n] = C[:, perm]
        rho = self.backend.density([C[k, :n] for k in range(3)], n)
        if perm is not None:  # the exchange works in the owned-then-ghost layout
            r = torch.empty_like(rho)
            r[perm] = rho
            rho = r
            C[:, perm] = C[:, :n].clone()
        self._mark("density")
        if not self.local_ghost_density:
            self.comm.exchange_rho(rho)
        self._mark("ghost_rho")
        self._note_work(C[0, :n_own], rho[:n_own])  # owned-then-ghost layout here in both modes
        if perm is not None:
            rho = rho[perm]
            C[:, :n] = C[:, perm]
        n_upd = n if perm is not None else n_own
        cols6 = [C[k, :n] for k in range(6)]
        if getattr(self.comm, "split", False):  # the zoned pass and split round 1, in sequence
            zones = self.geo.force_zones(self.reach)
            self.backend.force_step(cols6, rho, n, n_upd, zone=(1,) + zones)
            self.backend.force_step(cols6, rho, n, n_upd, zone=(2,) + zones)
            if perm is not None:
                C[:, perm] = C[:, :n].clone()
            self._mark("force")
            self.comm.exchange_begin()
            self.comm.exchange_end()
        else:
            self.backend.force_step(cols6, rho, n, n_upd)
            if perm is not None:
                C[:, perm] = C[:, :n].clone()
            self._mark("force")
            self.comm.exchange(migrate=True)
        self._mark("exchange")

    def _step_overlapped(self) -> None:
        """The step with both exchange rounds off the critical path.

        main stream:  density -> prepare (gather, zone lists) -> interior
                      force -> [wait payload] finish round 1
        side stream (high priority), after prepare: density round -> ghost
                      densities re-read -> boundary force -> round 1 begin
                      (selection, counts) -> payload (enqueued by the finish)
        Interior particles have no ghost neighbours and are not in any
        exchange list, so the interior force overlaps both rounds."""
        C = self.cols
        self._mark("start")
        n_own, n = self.n, self.n + self.ng
        rho = self.backend.density([C[k, :n] for k in range(3)], n)
        self._mark("density")
        self._note_work(C[0, :n_own], rho[:n_own])
        cols6 = [C[k, :n] for k in range(6)]
        zones = self.geo.force_zones(self.reach)
        self.backend.force_step(cols6, rho, n, n_own, zone=(3,) + zones)
        self._mark("prepare")
        main = torch.cuda.current_stream()
        if self._hp is None:
            self._hp = torch.cuda.Stream(device=main.device, priority=-1)
        self._hp.wait_stream(main)
        with torch.cuda.stream(self._hp):
            if not self.local_ghost_density:
                self.comm.exchange_rho(rho)
            self._mark_side("ghost_rho_done")
            self.backend.force_step(cols6, rho, n, n_own, zone=(1,) + zones)
            self._mark_side("boundary_done")
            self.comm.exchange_begin()
            self._mark_side("counts_done")
        self.backend.force_step(cols6, rho, n, n_own, zone=(2,) + zones)
        self._mark("force")
        self.comm.exchange_end()  # the main stream waits for the payload, which followed the boundary zone
        with torch.cuda.stream(self._hp):
            self._mark_side("payload_done")
        self._mark("exchange")
        rho.record_stream(self._hp)


def torch_classify(x, n, lo, hi, reach, flags):
    """forge_slab_classify with torch ops (CPU ranks in tests)."""
    x = x[:n]
    none = torch.zeros(n, dtype=torch.bool, device=x.device)
    halo, in_slab = bool(flags & 4), bool(flags & 8)
    left = (x < lo + reach if halo else x < lo) if flags & 1 else none
    right = (x >= hi - reach if halo else x >= hi) if flags & 2 else none
    if halo and in_slab:
        left = left & (x >= lo)
        right = right & (x < hi)
    both = none if halo else (left | right)
    return tuple(torch.nonzero(m).flatten() for m in (both, left, right))


def torch_compact(cols, n, gone):
    """forge_slab_compact with torch ops (CPU ranks in tests)."""
    k = gone.numel()
    if k == 0:
        return
    keep = n - k
    tail = torch.arange(keep, n, device=cols.device)
    fillers = tail[~torch.isin(tail, gone)]
    cols[:, gone[:fillers.numel()]] = cols[:, fillers]


class GpuBackend:
    """Per-rank compute through libforge_sph (sm_100a kernels)."""

    def __init__(self, forge_sph, cfg, capacity: int, device: int):
        self.f, self.cfg = forge_sph, cfg
        self.grid = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0.0, 0.0, 0.0), capacity, device)
        self.sp = forge_sph.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)
        stp = forge_sph.StepParams()
        stp.dt = cfg.dt
        stp.gravity[:] = list(cfg.gravity)
        stp.box_min[:] = list(cfg.box_min)
        stp.box_max[:] = list(cfg.box_max)
        stp.restitution = cfg.restitution
        stp.flags = 7
        self.stp = stp
        self.L = forge_sph.lib()
        self.capacity = capacity
        h = ctypes.c_void_p()
        forge_sph.check(self.L.forge_slab_create(capacity, device, ctypes.byref(h)))
        self.slab = h
        dev = torch.device("cuda", device)
        self.idx = torch.empty(2 * max(capacity, 1), dtype=torch.int32, device=dev)  # [A | L | R] <= 2n
        self.counts = torch.zeros(3, dtype=torch.int32, device=dev)

    def __del__(self):
        h = getattr(self, "slab", None)
        if h and self.f._lib is not None:
            self.f._lib.forge_slab_destroy(h)
            self.slab = None

    def classify(self, x, n, lo, hi, reach, flags):
        """(A, L, R) ascending index lists from forge_slab_classify (one
        device-to-host read of the three counts)."""
        self.f.check(self.L.forge_slab_classify(self.slab, x.data_ptr(), n, lo, hi, reach, flags,
                                                self.idx.data_ptr(), self.counts.data_ptr(), self._st()))
        a, l, r = self.counts.tolist()
        flat = self.idx[:a + l + r].long()
        return flat[:a], flat[a:a + l], flat[a + l:]

    def compact(self, cols, n, gone):
        if gone.numel() == 0:
            return
        g32 = gone.to(torch.int32)
        self.f.check(self.L.forge_slab_compact(cols.data_ptr(), cols.stride(0), cols.shape[0], n, g32.data_ptr(),
                                               gone.numel(), self._st()))

    def _st(self):
        return torch.cuda.current_stream().cuda_stream

    def density(self, pos, n):
        if n > self.capacity:
            raise self.f.ForgeError(self.f.FORGE_ERR_CAPACITY, f"{n} local particles > capacity {self.capacity}")
        rho = torch.empty(n, dtype=torch.float32, device=pos[0].device)
        self.f.check(self.L.forge_sph_density(self.grid.handle, ctypes.byref(self.sp), *(p.data_ptr() for p in pos),
                                              n, rho.data_ptr(), self._st()))
        return rho

    def force_step(self, cols, rho, n, n_update, zone=None):
        """Force + epilogue in place; rows >= n_update (ghosts) are skipped.
        zone = (mode, inner_lo, inner_hi, guard_lo, guard_hi) runs one half of
        the split pass (forge_sph_force_step_zone)."""
        if zone is None:
            self.f.check(self.L.forge_sph_force_step(self.grid.handle, ctypes.byref(self.sp),
                                                     ctypes.byref(self.stp), *(c.data_ptr() for c in cols),
                                                     rho.data_ptr(), n, n_update, self._st()))
            return
        z = self.f.ForceZone(*zone)
        self.f.check(self.L.forge_sph_force_step_zone(self.grid.handle, ctypes.byref(self.sp), ctypes.byref(self.stp),
                                                      *(c.data_ptr() for c in cols), rho.data_ptr(), n, n_update,
                                                      ctypes.byref(z), self._st()))
