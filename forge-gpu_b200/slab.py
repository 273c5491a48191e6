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
payloads), no data-path collective. The per-rank compute is a Backend:
GpuBackend runs the library's kernels (forge_sph_density,
forge_sph_force_step) on the rank's GPU; tests supply a CPU backend.
With ``order_by_id`` local arrays are kept in particle-id order, which makes
each particle's neighbour order, and hence the result, identical to the
single-device run.
"""
from __future__ import annotations

import ctypes

import torch

# Payload columns: x, y, z, vx, vy, vz, id (int32 bits carried in a float32).
_NCOL = 7


class SlabGeometry:
    """Uniform x-slabs of [x0, x1)."""

    def __init__(self, rank: int, world: int, x0: float, x1: float, h: float):
        self.rank, self.world, self.h = rank, world, h
        w = (x1 - x0) / world
        self.lo = x0 + w * rank
        self.hi = x0 + w * (rank + 1)
        self.first = rank == 0
        self.last = rank == world - 1

    def owned_mask(self, x: torch.Tensor) -> torch.Tensor:
        m = torch.ones_like(x, dtype=torch.bool)
        if not self.first:
            m &= x >= self.lo
        if not self.last:
            m &= x < self.hi
        return m


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
        ops = []
        for peer, t in sends.items():
            ops.append(self.dist.P2POp(self.dist.isend, t, peer))
        for peer, t in recvs.items():
            ops.append(self.dist.P2POp(self.dist.irecv, t, peer))
        if ops:
            for r in self.dist.batch_isend_irecv(ops):
                r.wait()

    def swap(self, to_left: torch.Tensor | None, to_right: torch.Tensor | None, ncol: int):
        """Send row blocks to rank-1 / rank+1, receive theirs. Returns
        (from_left, from_right), each (k, ncol) (empty where no neighbour)."""
        left = self.rank - 1 if self.rank > 0 else None
        right = self.rank + 1 if self.rank < self.world - 1 else None
        dt = torch.float32
        cnt = {}
        sends, recvs = {}, {}
        if left is not None:
            sends[left] = torch.tensor([to_left.shape[0]], dtype=torch.int64, device=self.device)
            cnt[left] = torch.zeros(1, dtype=torch.int64, device=self.device)
            recvs[left] = cnt[left]
        if right is not None:
            # distinct tensors per peer: a batch may not reuse one buffer
            sends[right] = torch.tensor([to_right.shape[0]], dtype=torch.int64, device=self.device)
            cnt[right] = torch.zeros(1, dtype=torch.int64, device=self.device)
            recvs[right] = cnt[right]
        self._p2p(sends, recvs)
        sends, recvs, out = {}, {}, {}
        for peer, blk in ((left, to_left), (right, to_right)):
            if peer is None:
                continue
            blk = blk.to(self.device)
            k = int(cnt[peer].item())
            out[peer] = torch.empty((k, ncol), dtype=dt, device=self.device)
            if k:
                recvs[peer] = out[peer]
            if blk.shape[0]:
                sends[peer] = blk.contiguous()
        self._p2p(sends, recvs)
        empty = torch.empty((0, ncol), dtype=dt, device=self.device)
        a, b = out.get(left, empty), out.get(right, empty)
        return a.to(self.home), b.to(self.home)


class SlabRun:
    """One rank's share of a sharded SPH run."""

    def __init__(self, dist, rank: int, world: int, cfg, pos, vel, backend, device: torch.device,
                 x_range=(0.0, 1.0), order_by_id: bool = False, comm_device=None):
        self.cfg, self.backend, self.device = cfg, backend, device
        self.geo = SlabGeometry(rank, world, x_range[0], x_range[1], cfg.h)
        self.ex = Exchanger(dist, rank, world, device, comm_device)
        self.order_by_id = order_by_id
        px = torch.as_tensor(pos[0])
        m = self.geo.owned_mask(px)
        ids = torch.arange(px.numel(), dtype=torch.int32)[m]
        cols = [torch.as_tensor(a)[m] for a in list(pos) + list(vel)]
        self.state = self._pack(cols, ids).to(device)  # (n_own, 7)
        self.last_halo = 0

    @staticmethod
    def _pack(cols, ids):
        return torch.stack(list(cols) + [ids.view(torch.float32)], dim=1).contiguous()

    @property
    def n_own(self) -> int:
        return self.state.shape[0]

    def ids(self) -> torch.Tensor:
        return self.state[:, 6].contiguous().view(torch.int32)

    def step(self) -> None:
        g, h = self.geo, self.cfg.h
        st = self.state
        x = st[:, 0]
        reach = h * (1.0 + 1e-5)
        left_idx = torch.nonzero(x < g.lo + reach).flatten() if not g.first else None
        right_idx = torch.nonzero(x >= g.hi - reach).flatten() if not g.last else None
        empty = st[:0]
        from_l, from_r = self.ex.swap(st[left_idx] if left_idx is not None else empty,
                                      st[right_idx] if right_idx is not None else empty, _NCOL)
        n_own, nl, nr = st.shape[0], from_l.shape[0], from_r.shape[0]
        self.last_halo = nl + nr
        local = torch.cat([st, from_l, from_r], dim=0)
        perm = None
        if self.order_by_id:
            perm = torch.argsort(local[:, 6].contiguous().view(torch.int32), stable=True)
            local = local[perm]
        cols = [local[:, k].contiguous() for k in range(6)]
        n = local.shape[0]
        rho = self.backend.density(cols[0:3], n)
        # ghost densities from their owners
        send_l = rho[_pos_after(perm, left_idx)].reshape(-1, 1) if left_idx is not None else rho[:0].reshape(0, 1)
        send_r = rho[_pos_after(perm, right_idx)].reshape(-1, 1) if right_idx is not None else rho[:0].reshape(0, 1)
        got_l, got_r = self.ex.swap(send_l, send_r, 1)
        ghost_rho = torch.cat([got_l.flatten(), got_r.flatten()])
        ghost_pos = torch.arange(n_own, n, device=rho.device)
        if perm is not None:
            inv = torch.empty_like(perm)
            inv[perm] = torch.arange(n, device=perm.device)
            ghost_pos = inv[ghost_pos]
        rho[ghost_pos] = ghost_rho
        # force + epilogue for owned particles only
        owned_flag = torch.zeros(n, dtype=torch.bool, device=rho.device)
        if perm is None:
            owned_flag[:n_own] = True
        else:
            owned_flag[perm < n_own] = True
        # owned rows lead the local arrays unless they were id-ordered
        self.backend.force_step(cols, rho, n, n_own if perm is None else n)
        new = torch.stack(cols + [local[:, 6]], dim=1)[owned_flag]
        # migration
        x = new[:, 0]
        go_l = (x < g.lo) if not g.first else torch.zeros_like(x, dtype=torch.bool)
        go_r = (x >= g.hi) if not g.last else torch.zeros_like(x, dtype=torch.bool)
        stay = ~(go_l | go_r)
        in_l, in_r = self.ex.swap(new[go_l], new[go_r], _NCOL)
        self.state = torch.cat([new[stay], in_l, in_r], dim=0).contiguous()
        if self.order_by_id:
            self.state = self.state[torch.argsort(self.ids(), stable=True)].contiguous()


def _pos_after(perm, idx):
    """Positions, in the (possibly id-ordered) local arrays, of owned rows idx."""
    if perm is None:
        return idx
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(perm.numel(), device=perm.device)
    return inv[idx]


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

    def _st(self):
        return torch.cuda.current_stream().cuda_stream

    def density(self, pos, n):
        if n > self.capacity:
            raise self.f.ForgeError(self.f.FORGE_ERR_CAPACITY, f"{n} local particles > capacity {self.capacity}")
        rho = torch.empty(n, dtype=torch.float32, device=pos[0].device)
        self.f.check(self.L.forge_sph_density(self.grid.handle, ctypes.byref(self.sp), *(p.data_ptr() for p in pos),
                                              n, rho.data_ptr(), self._st()))
        return rho

    def force_step(self, cols, rho, n, n_update):
        """Force + epilogue in place; rows >= n_update (ghosts) are skipped."""
        self.f.check(self.L.forge_sph_force_step(self.grid.handle, ctypes.byref(self.sp), ctypes.byref(self.stp),
                                                 *(c.data_ptr() for c in cols), rho.data_ptr(), n, n_update,
                                                 self._st()))
