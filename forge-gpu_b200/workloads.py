"""Seeded synthetic workloads for the particle hot path (host-side numpy).

The configurations restate BASELINE.json's five configs; the reference
publishes no dataset for them, so every input is generated here from a seed
(numpy PCG64). Choices the configs leave open are fixed here and stated:

* cfg0 "ref65k":   65,536 uniform points in [0,1)^3, h = cell = 0.025,
                   grid 40^3, mass 1.0, rho0 1000, k 3.0, mu 0.1,
                   velocities N(0, 0.01); trajectory steps use dt 1e-4,
                   gravity (0,-9.81,0), box [0,1]^3, restitution 1.0.
* cfg2 "dambreak1m": the config asks for 1M particles on a 0.5h lattice in
                   [0,0.4]x[0,0.8]x[0,0.4] with h = 0.025, which only holds
                   65,536. We keep the 1M, the 0.5h lattice (the SPH
                   resolution: 8 particles per cell, ~30 neighbours) and the
                   region, and scale h: N = 1,024,000 on an 80x160x80 lattice
                   at spacing 0.005, h = cell = 0.01, grid 100^3, dt 1e-4.
                   Two other readings are kept as workloads: the literal
                   h = 0.025 lattice ("dambreak65k", 65,536 particles) and
                   1M at h = 0.025 ("dambreak1m_h025": spacing h/5, 125
                   particles per cell, ~500 neighbours).
* cfg3 "sharded16m": 320x160x320 lattice at spacing h/2 in [0,1]x[0,0.5]x[0,1],
                   h = 0.00625, grid 160^3, dt 2.5e-5.
* cfg4 "blobs4m":  4,194,304 points from 64 Gaussian blobs (centres uniform
                   in [0.1,0.9]^3, sigma 0.02), h = 0.0125, grid 80^3, dt 5e-5.
Lattice configs use mass = rho0 * spacing^3 (rest density at rest); blobs
use mass = rho0 / N (unit volume). Velocities start at zero except cfg0.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

SEED = 0x5EED


@dataclass
class SphConfig:
    name: str
    n: int
    h: float
    cell_size: float
    dims: tuple
    mass: float
    rest_density: float = 1000.0
    gas_constant: float = 3.0
    viscosity: float = 0.1
    dt: float = 1e-4
    gravity: tuple = (0.0, -9.81, 0.0)
    box_min: tuple = (0.0, 0.0, 0.0)
    box_max: tuple = (1.0, 1.0, 1.0)
    restitution: float = 1.0
    steps: int = 1

    @property
    def cells(self) -> int:
        return self.dims[0] * self.dims[1] * self.dims[2]

    @property
    def key_bits(self) -> int:
        return max(1, int(self.cells - 1).bit_length())


def _lattice(nx, ny, nz, spacing, lo=(0.0, 0.0, 0.0)):
    z, y, x = np.meshgrid(np.arange(nz, dtype=np.float32), np.arange(ny, dtype=np.float32),
                          np.arange(nx, dtype=np.float32), indexing="ij")
    s = np.float32(spacing)
    half = np.float32(0.5)
    px = (np.float32(lo[0]) + (x.ravel() + half) * s).astype(np.float32)
    py = (np.float32(lo[1]) + (y.ravel() + half) * s).astype(np.float32)
    pz = (np.float32(lo[2]) + (z.ravel() + half) * s).astype(np.float32)
    return px, py, pz


def config(name: str) -> SphConfig:
    if name == "ref65k":
        return SphConfig(name, 65536, 0.025, 0.025, (40, 40, 40), 1.0, steps=100)
    if name == "dambreak1m":
        s = 0.01 / 2
        return SphConfig(name, 80 * 160 * 80, 0.01, 0.01, (100, 100, 100), 1000.0 * s ** 3, steps=1000)
    if name == "dambreak1m_h025":
        s = 0.025 / 5
        return SphConfig(name, 80 * 160 * 80, 0.025, 0.025, (40, 40, 40), 1000.0 * s ** 3, steps=1000)
    if name == "dambreak65k":
        s = 0.025 / 2
        return SphConfig(name, 32 * 64 * 32, 0.025, 0.025, (40, 40, 40), 1000.0 * s ** 3, steps=1000)
    if name == "sharded16m":
        s = 0.00625 / 2
        return SphConfig(name, 320 * 160 * 320, 0.00625, 0.00625, (160, 160, 160), 1000.0 * s ** 3, dt=2.5e-5,
                         steps=200)
    if name == "blobs4m":
        return SphConfig(name, 4194304, 0.0125, 0.0125, (80, 80, 80), 1000.0 / 4194304, dt=5e-5, steps=100)
    raise KeyError(name)


def small(name: str, n: int, dims=(16, 16, 16)) -> SphConfig:
    """A scaled-down config with the same occupancy model, for parity tests."""
    c = config(name)
    c.n = n
    c.dims = dims
    c.cell_size = c.h = 1.0 / dims[0]
    return c


def particles(cfg: SphConfig, seed: int = SEED):
    """(pos, vel): lists of three float32 numpy arrays, original order."""
    rng = np.random.Generator(np.random.PCG64(seed))
    n = cfg.n
    if cfg.name in ("ref65k",):
        pos = [rng.random(n, dtype=np.float32) for _ in range(3)]
        vel = [rng.normal(0.0, 0.01, n).astype(np.float32) for _ in range(3)]
        return pos, vel
    if cfg.name in ("dambreak1m", "dambreak1m_h025"):
        pos = list(_lattice(80, 160, 80, 0.005))
    elif cfg.name == "dambreak65k":
        pos = list(_lattice(32, 64, 32, 0.025 / 2))
    elif cfg.name == "sharded16m":
        pos = list(_lattice(320, 160, 320, 0.00625 / 2))
    elif cfg.name == "blobs4m":
        nb = 64
        centres = rng.uniform(0.1, 0.9, (nb, 3)).astype(np.float32)
        per = n // nb
        g = rng.normal(0.0, 0.02, (n, 3)).astype(np.float32)
        b = np.repeat(np.arange(nb), per)
        xyz = centres[b] + g
        pos = [np.ascontiguousarray(xyz[:, a]) for a in range(3)]
    else:
        raise KeyError(cfg.name)
    if pos[0].size != n:  # scaled-down variants: uniform points in the cfg's box
        pos = [rng.random(n, dtype=np.float32) for _ in range(3)]
    vel = [np.zeros(n, np.float32) for _ in range(3)]
    return pos, vel


def uniform_particles(n: int, seed: int = SEED, lo=0.0, hi=1.0, vsigma=0.01):
    rng = np.random.Generator(np.random.PCG64(seed))
    pos = [(np.float32(lo) + np.float32(hi - lo) * rng.random(n, dtype=np.float32)).astype(np.float32)
           for _ in range(3)]
    vel = [rng.normal(0.0, vsigma, n).astype(np.float32) for _ in range(3)]
    return pos, vel


def sort_keys(kind: str, n: int, seed: int = SEED) -> np.ndarray:
    """cfg1 keys: 'uniform' u32 or 'morton' 30-bit Morton codes."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if kind == "uniform":
        return rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    if kind == "morton":
        xyz = np.floor(rng.random((n, 3), dtype=np.float32) * np.float32(1024)).astype(np.uint32)
        return morton30(xyz[:, 0], xyz[:, 1], xyz[:, 2])
    raise KeyError(kind)


def _spread10(v):
    v = v.astype(np.uint32) & np.uint32(0x3FF)
    v = (v | (v << np.uint32(16))) & np.uint32(0x030000FF)
    v = (v | (v << np.uint32(8))) & np.uint32(0x0300F00F)
    v = (v | (v << np.uint32(4))) & np.uint32(0x030C30C3)
    v = (v | (v << np.uint32(2))) & np.uint32(0x09249249)
    return v


def morton30(x, y, z):
    return (_spread10(x) | (_spread10(y) << np.uint32(1)) | (_spread10(z) << np.uint32(2))).astype(np.uint32)
