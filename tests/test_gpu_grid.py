"""GPU parity: hash-grid build (cell hash, stable sort, cell-start table)
and the batched neighbour query, bit-exact against the oracle."""
import json
import os

import numpy as np
import pytest

import forge_sph
import oracle
import workloads
from _util import dev, host_u32

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def build_and_compare(torch, pos, cs, dims, origin=(0.0, 0.0, 0.0)):
    n = pos[0].size
    g = forge_sph.HashGrid(cs, dims, origin, max(n, 1), 0)
    g.build(tuple(dev(torch, p) for p in pos))
    g.check()
    ci, si, cst = oracle.grid_build(*pos, cs, dims, origin)
    assert np.array_equal(host_u32(g.cell_indices)[:n], ci)
    assert np.array_equal(host_u32(g.sorted_indices)[:n], si)
    assert np.array_equal(host_u32(g.cell_start), cst)
    return g


def test_cfg0_grid_build_bit_exact(cuda):
    cfg = workloads.config("ref65k")
    pos, _ = workloads.particles(cfg)
    build_and_compare(cuda, pos, cfg.cell_size, cfg.dims)


@pytest.mark.parametrize("n", [0, 1, 2, 4095, 4097, 100_000])
def test_ragged_sizes_with_outside_points(cuda, n):
    pos, _ = workloads.uniform_particles(n, seed=n, lo=-0.2, hi=1.3)
    build_and_compare(cuda, pos, 0.05, (20, 17, 23), origin=(0.0, 0.0, 0.0))


def test_origin_and_non_finite_positions(cuda):
    pos, _ = workloads.uniform_particles(10_000, seed=9, lo=-1.0, hi=2.0)
    pos[0][:5] = [np.nan, np.inf, -np.inf, 1e30, -1e30]
    pos[1][5:8] = np.nan
    build_and_compare(cuda, pos, 0.1, (16, 8, 12), origin=(-0.5, 0.25, -0.125))


def test_all_particles_in_one_cell(cuda):
    n = 70_000
    pos = [np.full(n, 0.51, np.float32) for _ in range(3)]
    build_and_compare(cuda, pos, 0.1, (10, 10, 10))


def test_aos_build_matches_soa(cuda):
    k = GOLD["hashgrid_uniform"]
    xyz = np.array(k["positions"], np.float32)
    g = forge_sph.HashGrid(k["cell_size"], k["dims"], k["origin"], xyz.shape[0], 0)
    g.build(cuda.from_numpy(xyz).cuda())
    ci, si, cst = oracle.grid_build_aos(xyz, k["cell_size"], k["dims"], k["origin"])
    n = xyz.shape[0]
    assert np.array_equal(host_u32(g.cell_indices)[:n], ci)
    assert np.array_equal(host_u32(g.sorted_indices)[:n], si)
    assert np.array_equal(host_u32(g.cell_start), cst)


def test_hashgrid_kats_query(cuda):
    # tests/hashgrid_test.rs:6-36 and :38-88
    k = GOLD["hashgrid_basic"]
    g = forge_sph.HashGrid(k["cell_size"], k["dims"], k["origin"], 100, 0)
    g.build(cuda.tensor(k["positions"], dtype=cuda.float32))
    hits = g.query_neighbors(k["query"], k["radius"])
    assert all(j in hits for j in k["must_contain"])
    assert all(j not in hits for j in k["must_not_contain"])
    k = GOLD["hashgrid_uniform"]
    g = forge_sph.HashGrid(k["cell_size"], k["dims"], k["origin"], 1000, 0)
    xyz = np.array(k["positions"], np.float32)
    g.build(cuda.from_numpy(xyz).cuda())
    hits = g.query_neighbors(k["query"], k["radius"])
    assert len(hits) >= k["min_hits"]
    ci, si, cst = oracle.grid_build_aos(xyz, k["cell_size"], k["dims"], k["origin"])
    expect = oracle.query(xyz[:, 0], xyz[:, 1], xyz[:, 2], cst, si, k["cell_size"], k["dims"], k["query"],
                          k["radius"], k["origin"])
    assert hits == expect.tolist()


def test_batched_query_vs_oracle(cuda):
    n, nq = 20_000, 3000
    cs, dims = 0.05, (20, 20, 20)
    pos, _ = workloads.uniform_particles(n, seed=21)
    q, _ = workloads.uniform_particles(nq, seed=22, lo=-0.1, hi=1.1)
    g = forge_sph.HashGrid(cs, dims, (0, 0, 0), n, 0)
    g.build(tuple(dev(cuda, p) for p in pos))
    counts, offsets, hits = g.query_batch(*(dev(cuda, a) for a in q), 0.05)
    counts, offsets, hits = host_u32(counts), host_u32(offsets), host_u32(hits)
    ci, si, cst = oracle.grid_build(*pos, cs, dims)
    for i in range(nq):
        e = oracle.query(*pos, cst, si, cs, dims, (q[0][i], q[1][i], q[2][i]), 0.05)
        assert counts[i] == e.size
        assert np.array_equal(hits[offsets[i]:offsets[i + 1]], e), i


def test_sharded16m_full_size_grid_bit_exact(cuda):
    """cfg3 at full size: 16,384,000 particles, 160^3 cells (22-bit keys,
    3 sort passes) -- the size where the reference's scan breaks."""
    cfg = workloads.config("sharded16m")
    pos, _ = workloads.particles(cfg)
    build_and_compare(cuda, pos, cfg.cell_size, cfg.dims)


def test_blobs4m_full_size_grid_bit_exact(cuda):
    cfg = workloads.config("blobs4m")
    pos, _ = workloads.particles(cfg)
    build_and_compare(cuda, pos, cfg.cell_size, cfg.dims)


def test_build_is_deterministic(cuda):
    cfg = workloads.config("ref65k")
    pos, _ = workloads.particles(cfg)
    g = forge_sph.HashGrid(cfg.cell_size, cfg.dims, (0, 0, 0), cfg.n, 0)
    t = tuple(dev(cuda, p) for p in pos)
    g.build(t)
    a = host_u32(g.sorted_indices).copy()
    for _ in range(3):
        g.build(t)
        assert np.array_equal(host_u32(g.sorted_indices), a)


def test_query_points_on_the_radius(cuda):
    """Particles placed on spheres of the query radius around each query
    point, so dist^2 lands within an ulp or two of r^2: the <= test must be
    decided with every operation rounded, as hashgrid.rs:183-184 does (an
    FMA-contracted dist^2 flips some of these)."""
    rng = np.random.default_rng(77)
    nq, per = 200, 64
    cs, dims, radius = 0.05, (20, 20, 20), 0.05
    q = rng.uniform(0.1, 0.9, (nq, 3)).astype(np.float32)
    u = rng.normal(size=(nq, per, 3))
    u /= np.linalg.norm(u, axis=2, keepdims=True)
    p = (q[:, None, :].astype(np.float64) + radius * u).astype(np.float32).reshape(-1, 3)
    pos = [np.ascontiguousarray(p[:, k]) for k in range(3)]
    qs = [np.ascontiguousarray(q[:, k]) for k in range(3)]
    g = forge_sph.HashGrid(cs, dims, (0, 0, 0), p.shape[0], 0)
    g.build(tuple(dev(cuda, a) for a in pos))
    counts, offsets, hits = g.query_batch(*(dev(cuda, a) for a in qs), radius)
    counts, offsets, hits = host_u32(counts), host_u32(offsets), host_u32(hits)
    ci, si, cst = oracle.grid_build(*pos, cs, dims)
    on_edge = 0
    for i in range(nq):
        e = oracle.query(*pos, cst, si, cs, dims, (qs[0][i], qs[1][i], qs[2][i]), radius)
        assert np.array_equal(hits[offsets[i]:offsets[i + 1]], e), i
        on_edge += per - int(np.count_nonzero((e >= i * per) & (e < (i + 1) * per)))
    assert 0 < on_edge < nq * per  # the case really straddles the radius
