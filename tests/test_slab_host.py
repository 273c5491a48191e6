"""Host logic of the sharded step (no GPU, no process group): slab bounds,
load-balancing bounds, the split force pass's zones."""
import numpy as np
import pytest

import slab


def test_uniform_and_explicit_bounds():
    g = slab.SlabGeometry(2, 4, 0.0, 1.0, 0.01)
    assert (g.lo, g.hi, g.first, g.last) == (0.5, 0.75, False, False)
    g = slab.SlabGeometry(0, 3, 0.0, 1.0, 0.01, bounds=[0.0, 0.2, 0.7, 1.0])
    assert (g.lo, g.hi, g.first) == (0.0, 0.2, True)


def test_quantile_bounds_split_counts_evenly():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.normal(0.2, 0.03, 30000), rng.normal(0.8, 0.05, 10000)]).clip(0, 0.999)
    hist = np.histogram(x, bins=4096, range=(0.0, 1.0))[0]
    b = slab.quantile_bounds(hist, 0.0, 1.0, 4)
    assert b[0] == 0.0 and b[-1] == 1.0 and all(b[k] < b[k + 1] for k in range(4))
    counts = np.histogram(x, bins=b)[0]
    assert counts.max() - counts.min() <= 0.01 * x.size, counts


def test_quantile_bounds_empty_histogram_is_uniform():
    assert slab.quantile_bounds(np.zeros(16), 0.0, 1.0, 4) == [0.0, 0.25, 0.5, 0.75, 1.0]


def test_balanced_bounds_move_at_most_one_slab_and_keep_min_width():
    old = [0.0, 0.25, 0.5, 0.75, 1.0]
    hist = np.zeros(1000)
    hist[100:150] = 1.0  # everything in [0.1, 0.15): the quantiles want all bounds there
    new = slab.balanced_bounds(hist, 0.0, 1.0, old, 0.02)
    for k in range(1, 4):
        assert old[k - 1] <= new[k] <= old[k + 1]
    assert all(new[k + 1] - new[k] >= 0.02 * (1 - 1e-6) for k in range(4))
    assert new != old
    # float32 values: what the library compares with
    assert all(float(np.float32(v)) == v for v in new)


def test_balanced_bounds_keep_old_when_min_width_cannot_hold():
    old = [0.0, 0.3, 0.6, 1.0]
    hist = np.ones(100)
    assert slab.balanced_bounds(hist, 0.0, 1.0, old, 0.5) == old


def test_min_width_bounds():
    b = slab.min_width_bounds([0.0, 0.001, 0.002, 1.0], 0.1)
    assert all(b[k + 1] - b[k] >= 0.1 - 1e-6 for k in range(3))


@pytest.mark.parametrize("rank,world", [(0, 3), (1, 3), (2, 3)])
def test_force_zones_guard_and_margin(rank, world):
    h = 0.00625
    g = slab.SlabGeometry(rank, world, 0.0, 1.0, h)
    reach = h * (1 + 1e-5)
    inner_lo, inner_hi, guard_lo, guard_hi = g.force_zones(reach)
    f32 = np.float32
    if g.first:
        assert inner_lo == guard_lo == -np.inf
    else:  # the guard is the classification's own float32 sum lo + reach
        assert guard_lo == float(f32(g.lo) + f32(reach))
        assert inner_lo == float(f32(guard_lo) + f32(h / 4))
    if g.last:
        assert inner_hi == guard_hi == np.inf
    else:
        assert guard_hi == float(f32(g.hi) - f32(reach))
        assert inner_hi < guard_hi


def test_halo_width_is_one_or_two():
    import torch
    import workloads
    cfg = workloads.small("ref65k", 100, (8, 8, 8))
    pos, vel = workloads.uniform_particles(cfg.n, seed=1)
    with pytest.raises(ValueError, match="halo_width"):
        slab.SlabRun(None, 0, 1, cfg, pos, vel, None, torch.device("cpu"), halo_width=1.5)


@pytest.mark.parametrize("world,halo_width,ok", [(4, 1.0, True), (4, 2.0, False), (8, 1.0, False)])
def test_uniform_slabs_narrower_than_two_reaches_are_rejected(world, halo_width, ok):
    """h = 1/16: 4 slabs of 0.25 hold a 1h halo (2 * reach = 0.125) but not a
    2h one (2 * reach = 0.25 + 1e-5 rounding margin); 8 slabs of 0.125 hold
    neither. A halo never skips a rank, so too-narrow slabs must fail loudly."""
    import torch
    import workloads
    cfg = workloads.small("ref65k", 200, (16, 16, 16))
    pos, vel = workloads.uniform_particles(cfg.n, seed=3)
    made = []

    class _Comm:  # stands in for the exchange: only construction is tested
        def __init__(self, run):
            made.append(run)

        def exchange(self, migrate):
            pass

    if ok:
        slab.SlabRun(None, 1, world, cfg, pos, vel, None, torch.device("cpu"), halo_width=halo_width, comm=_Comm)
        assert made
    else:
        with pytest.raises(ValueError, match="2 \\* reach"):
            slab.SlabRun(None, 1, world, cfg, pos, vel, None, torch.device("cpu"), halo_width=halo_width,
                         comm=_Comm)
