"""Failure detection of the sharded step, on CPU ranks run as threads over
an in-process mailbox transport (slab_cpu.MailboxHub) with injected delays,
dropped messages and a rank that dies: no GPU and no real process group.

With random delays the trajectory is still the single-process one bit for
bit; a dropped message or a dead rank makes its neighbours raise
ExchangeTimeout within the transport's timeout instead of hanging."""
import threading
import time

import numpy as np
import torch

import oracle
import slab
import slab_cpu
import workloads
from test_slab_gloo import OracleBackend, _cfg, _inputs

STEPS = 6


def _run_threads(world, hub, steps, die_at=None):
    """Runs `world` ranks as threads; returns per-rank (state or exception)."""
    out = [None] * world
    cfg = _cfg()
    pos, vel = _inputs(cfg)

    def main(r):
        try:
            run = slab.SlabRun(hub.rank(r), r, world, cfg, pos, vel, OracleBackend(cfg), torch.device("cpu"),
                               order_by_id=True, comm=lambda run: slab_cpu.PyComm(run, hub.rank(r)))
            for s in range(steps):
                if die_at is not None and die_at == (r, s):
                    raise SystemExit(f"rank {r} stops at step {s}")
                run.step()
            out[r] = run.state.numpy().copy()
        except BaseException as e:  # noqa: BLE001 -- recorded for the test
            out[r] = e

    th = [threading.Thread(target=main, args=(r,), daemon=True) for r in range(world)]
    t0 = time.monotonic()
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=120)
    assert not any(t.is_alive() for t in th), "a rank hung"
    return out, time.monotonic() - t0


def test_delayed_messages_keep_the_trajectory_exact():
    hub = slab_cpu.MailboxHub(3, timeout=30.0, delay=(0.0, 0.003), seed=1)
    out, _ = _run_threads(3, hub, STEPS)
    for o in out:
        assert isinstance(o, np.ndarray), o
    rows = np.concatenate(out)
    ids = rows[:, 6].copy().view(np.int32)
    cfg = _cfg()
    assert np.array_equal(np.sort(ids), np.arange(cfg.n))
    pos, vel = _inputs(cfg)
    sp = oracle.StepParams(cfg.dt, cfg.gravity, cfg.box_min, cfg.box_max, cfg.restitution, 7)
    p = oracle.SphParams(cfg.h, cfg.mass, cfg.gas_constant, cfg.rest_density, cfg.viscosity)
    for _ in range(STEPS):
        oracle.step(p, sp, pos, vel, cfg.cell_size, cfg.dims)
    assert np.array_equal(rows[np.argsort(ids), :6], np.stack(pos + vel, axis=1))


def test_dropped_message_is_detected_by_timeout():
    # drop the 5th message rank 1 sends to rank 0 (mid-run: round 1 of step 1)
    hub = slab_cpu.MailboxHub(3, timeout=1.0, drop=lambda src, dst, seq: (src, dst, seq) == (1, 0, 4))
    out, took = _run_threads(3, hub, STEPS)
    assert isinstance(out[0], slab_cpu.ExchangeTimeout), out[0]
    assert "from rank 1" in str(out[0])
    assert any(isinstance(o, slab_cpu.ExchangeTimeout) for o in out[1:]), "the failure did not propagate"
    assert took < 60


def test_dead_rank_is_detected_by_its_neighbours():
    hub = slab_cpu.MailboxHub(3, timeout=1.0)
    out, took = _run_threads(3, hub, STEPS, die_at=(2, 3))
    assert isinstance(out[2], SystemExit)
    assert isinstance(out[1], slab_cpu.ExchangeTimeout) and "from rank 2" in str(out[1]), out[1]
    assert isinstance(out[0], slab_cpu.ExchangeTimeout), out[0]  # rank 1 stopped answering too
    assert took < 60


def test_rebalance_all_reduce_over_mailbox():
    """The rebalancing all-reduce over the mailbox: every rank gets the same
    bounds; a missing rank turns into ExchangeTimeout."""
    hub = slab_cpu.MailboxHub(2, timeout=1.0)
    got = [None, None]

    def main(r):
        t = torch.full((4,), float(r + 1))
        hub.rank(r).all_reduce(t)
        got[r] = t.tolist()

    th = [threading.Thread(target=main, args=(r,)) for r in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert got == [[3.0] * 4, [3.0] * 4]
    lone = slab_cpu.MailboxHub(2, timeout=0.5)
    try:
        lone.rank(0).all_reduce(torch.ones(2))
        raise AssertionError("expected ExchangeTimeout")
    except slab_cpu.ExchangeTimeout:
        pass
