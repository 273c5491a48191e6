"""CPU-rank plumbing for the slab-decomposition tests (not part of the
library): the two exchange rounds of forge-gpu_b200/slab.py in Python over
torch.distributed (gloo) or an in-process mailbox with injected faults, and
torch restatements of the library's selection and compaction kernels.

The library's own exchange (slab.NcclComm, forge_slab_exchange*) runs the same
protocol inside libforge_sph over NCCL; these stand in for it on CPU ranks.
"""
from __future__ import annotations

import torch

_NCOL = 7


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


def torch_x_hist(x, w, lo, hi, bins):
    """forge_slab_x_hist with torch ops (CPU ranks in tests)."""
    idx = ((x.double() - lo) * (bins / (hi - lo))).floor().clamp_(0, bins - 1).long()
    return torch.bincount(idx, weights=None if w is None else w.double().clamp(min=0), minlength=bins).double()
