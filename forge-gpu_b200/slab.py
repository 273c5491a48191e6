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
forge_sph_force_step[_zone]) on the rank's GPU; the tests supply a CPU
backend and CPU-rank transports of their own.
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
    rounds in the library (GPU ranks, NCCL).
    """

    def __init__(self, dist, rank: int, world: int, cfg, pos, vel, backend, device: torch.device,
                 x_range=(0.0, 1.0), order_by_id: bool = False, capacity: int | None = None,
                 comm="nccl", forge_sph=None, balance: bool = False, hist_bins: int = 4096,
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
        self.check_widths(self.geo.bounds)
        self._set_window()
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
        # "nccl": both rounds inside the library over its own NCCL communicator;
        # otherwise a factory comm(run) of an object with the same methods
        # (exchange, set_bounds, exchange_rho) -- the tests' CPU-rank transport
        self.comm = NcclComm(self, dist, forge_sph) if comm == "nccl" else comm(self)
        self.comm.exchange(migrate=False)  # initial halo

    def _set_window(self) -> None:
        """Shrinks the backend's grid to this slab along x (owned particles,
        ghosts within reach of a face, and one cell each side for the ghosts'
        neighbours), so the cell table scales with the shard."""
        if hasattr(self.backend, "set_window"):
            g = self.geo
            lo = -np.inf if g.first else g.lo - self.reach
            hi = np.inf if g.last else g.hi + self.reach
            self.backend.set_window(lo, hi)

    def check_widths(self, bounds) -> None:
        """Every slab must be at least 2 * reach wide: halo and migrant lists
        only go to the adjacent ranks, so a narrower slab would let a ghost
        two ranks away go missing (silently wrong densities and forces)."""
        w = [bounds[k + 1] - bounds[k] for k in range(len(bounds) - 1)]
        need = 2.0 * self.reach
        if min(w) < need * (1 - 1e-6):
            k = int(np.argmin(w))
            raise ValueError(f"slab {k} is {w[k]:.6g} wide, below 2 * reach = {need:.6g} (h = {self.cfg.h}, "
                             f"halo width {self.reach / self.cfg.h:.3g} h): use fewer ranks or halo_width 1")

    def _x_hist(self, x: torch.Tensor, w: torch.Tensor | None) -> torch.Tensor:
        """hist_bins-bin histogram of x over x_range (weights w, or counts),
        computed by the backend (forge_slab_x_hist on GPU ranks)."""
        lo, hi = self.x_range
        return self.backend.x_hist(x, w, lo, hi, self.hist_bins)

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
        self.check_widths(new)
        self.geo.set_bounds(new)
        self._set_window()
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

        main stream:  density -> prepare (gather, zone lists) -> [wait for
                      the ghost densities] -> boundary force -> interior
                      force -> [wait payload] finish round 1
        side stream (high priority): density round (beside the prepare
                      step), then, once the boundary force is done, round 1
                      begin (selection, counts) and the payload (enqueued by
                      the finish) -- beside the interior force.
        The boundary force runs alone on the GPU (it is short and everything
        after it waits for it); interior particles have no ghost neighbours
        and are in no exchange list, so the interior force, the bulk of the
        step, overlaps all of round 1."""
        C = self.cols
        self._mark("start")
        n_own, n = self.n, self.n + self.ng
        rho = self.backend.density([C[k, :n] for k in range(3)], n)
        self._mark("density")
        self._note_work(C[0, :n_own], rho[:n_own])
        cols6 = [C[k, :n] for k in range(6)]
        zones = self.geo.force_zones(self.reach)
        main = torch.cuda.current_stream()
        if self._hp is None:
            self._hp = torch.cuda.Stream(device=main.device, priority=-1)
        if not self.local_ghost_density:
            self._hp.wait_stream(main)
            with torch.cuda.stream(self._hp):
                self.comm.exchange_rho(rho)
        self.backend.force_step(cols6, rho, n, n_own, zone=(3,) + zones)
        self._mark("prepare")
        main.wait_stream(self._hp)  # the ghosts' exact densities
        self.backend.force_step(cols6, rho, n, n_own, zone=(1,) + zones)
        self._mark("boundary")
        self._hp.wait_stream(main)
        with torch.cuda.stream(self._hp):
            self.comm.exchange_begin()
            self._mark_side("counts_done")
        self.backend.force_step(cols6, rho, n, n_own, zone=(2,) + zones)
        self._mark("force")
        self.comm.exchange_end()  # the main stream waits for the payload
        with torch.cuda.stream(self._hp):
            self._mark_side("payload_done")
        self._mark("exchange")
        rho.record_stream(self._hp)


class GpuBackend:
    """Per-rank compute through libforge_sph (sm_100a kernels)."""

    def __init__(self, forge_sph, cfg, capacity: int, device: int, walk: int = 0):
        self.f, self.cfg = forge_sph, cfg
        self.grid = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0.0, 0.0, 0.0), capacity, device)
        self.grid.set_walk(walk)  # neighbour-pass kernel family (0: by particle count)
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

    def set_window(self, x_lo: float, x_hi: float) -> None:
        """Grid x-window covering positions [x_lo, x_hi) plus one cell each
        side (infinite bounds: to the grid's edge)."""
        cs, nx = self.cfg.cell_size, self.cfg.dims[0]
        c0 = 0 if not np.isfinite(x_lo) else max(0, int(np.floor(x_lo / cs)) - 1)
        c1 = nx - 1 if not np.isfinite(x_hi) else min(nx - 1, int(np.floor(x_hi / cs)) + 1)
        self.grid.set_x_window(c0, c1 - c0 + 1)

    def classify(self, x, n, lo, hi, reach, flags):
        """(A, L, R) ascending index lists from forge_slab_classify (one
        device-to-host read of the three counts)."""
        self.f.check(self.L.forge_slab_classify(self.slab, x.data_ptr(), n, lo, hi, reach, flags,
                                                self.idx.data_ptr(), self.counts.data_ptr(), self._st()))
        a, l, r = self.counts.tolist()
        flat = self.idx[:a + l + r].long()
        return flat[:a], flat[a:a + l], flat[a + l:]

    def x_hist(self, x, w, lo, hi, bins):
        """forge_slab_x_hist: fixed-point, order-independent x-histogram."""
        out = torch.empty(bins, dtype=torch.float64, device=x.device)
        self.f.check(self.L.forge_slab_x_hist(self.slab, x.data_ptr(), None if w is None else w.data_ptr(),
                                              x.numel(), lo, hi, bins, out.data_ptr(), self._st()))
        return out

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
