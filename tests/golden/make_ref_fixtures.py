"""Writes tests/golden/ref_sph.npz: outputs of the reference's OWN SPH and
per-particle kernels, run on the host, on small seeded cases.

The kernels are the reference's CUDA C strings, extracted verbatim by
oracle/ref_extract.py and built by `make -C oracle ref` into
oracle/_ref/libref.so (git-ignored), one function call per CUDA thread:

  grid build  compute_cell_index / count_cells / scatter_particles / set_last
              (sph_density.rs:72-122, :342), serial in thread order
  density     sph_density (sph_density.rs:401-461)
  pressure    sph_pressure (sph_pressure.rs:28-112)
  viscosity   sph_viscosity (sph_viscosity.rs:27-106)
  modules     gravity.rs:31-34, drag.rs:18-20, integrate.rs:16-31,
              ground_plane.rs:19-21, sphere_collider.rs:22-41,
              box_collider.rs:26-47

pressure/viscosity update velocities in place; they are run in Jacobi form
(each particle's thread sees the unmodified input velocities), the form this
library implements. Pressure runs on zero velocities with dt = 1, so its
output is its acceleration; viscosity on the case's velocities with dt = 1.

Inputs are stored beside the outputs, so the fixtures do not depend on a
generator. Run from the repository root (needs a reference checkout):
    make -C oracle ref && python tests/golden/make_ref_fixtures.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import ref  # noqa: E402

PHYS = dict(h=0.025, mass=1.0, k=3.0, rho0=1000.0, mu=0.1)


def digest(*arrays) -> str:
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()


def cases():
    rng = np.random.Generator(np.random.PCG64(2026))
    out = {}
    # cfg0's occupancy (65,536 per unit cube) on a 0.4^3 box, 16^3 cells
    n = 4096
    pos = rng.random((3, n), dtype=np.float32) * np.float32(0.4)
    vel = rng.normal(0.0, 0.01, (3, n)).astype(np.float32)
    out["cube4k"] = dict(pos=pos, vel=vel, cs=0.025, dims=(16, 16, 16), mass=1.0)
    # edge cases: points outside the grid (clamped to border cells), a dense
    # clump, exact duplicates (r = 0: skipped by the force terms, counted
    # by density), points on cell faces
    n1 = 1500
    p = rng.uniform(-0.05, 0.45, (3, n1)).astype(np.float32)
    clump = (np.float32(0.2) + rng.normal(0.0, 0.004, (3, 400))).astype(np.float32)
    dup = p[:, :50].copy()
    faces = (np.float32(0.025) * rng.integers(0, 16, (3, 200))).astype(np.float32)
    pos = np.ascontiguousarray(np.concatenate([p, clump, dup, faces], axis=1))
    vel = rng.normal(0.0, 0.05, pos.shape).astype(np.float32)
    out["edges"] = dict(pos=pos, vel=vel, cs=0.025, dims=(16, 16, 16), mass=1.0)
    # a mass so small that isolated particles fall below rho = 1e-6 (self
    # term 315/(64 pi h^3) * m ~ 3e-7) while clumped ones do not: the
    # reference's rho < 1e-6 skip rules on both sides of a pair
    out["lowmass"] = dict(pos=out["edges"]["pos"], vel=out["edges"]["vel"], cs=0.025, dims=(16, 16, 16),
                          mass=3e-12)
    return out


def run_case(c):
    pos = [np.ascontiguousarray(c["pos"][k]) for k in range(3)]
    vel = [np.ascontiguousarray(c["vel"][k]) for k in range(3)]
    ph = dict(PHYS, mass=c["mass"])
    ci, si, cst = ref.grid_build(pos, c["cs"], c["dims"])
    rho = ref.density(pos, cst, si, ph["h"], ph["mass"], c["cs"], c["dims"])
    zero = [np.zeros_like(v) for v in vel]
    pa = ref.pressure(pos, zero, rho, cst, si, ph["h"], ph["mass"], ph["k"], ph["rho0"], c["cs"], c["dims"], 1.0)
    vv = ref.viscosity(pos, vel, rho, cst, si, ph["h"], ph["mass"], ph["mu"], c["cs"], c["dims"], 1.0)
    return dict(cell_idx=ci, sorted_idx=si, cell_start=cst, density=rho, pressure_accel=np.stack(pa),
                viscosity_vel=np.stack(vv))


OPS = [(1, (0.0, -9.81, 0.0)), (2, (0.5,)), (3, ()), (4, (0.05, 0.6)), (5, (0.5, 0.5, 0.5, 0.2, 0.8)),
       (6, (0.0, 0.0, 0.0, 1.0, 1.0, 1.0, 0.9))]


def epilogue_case():
    rng = np.random.Generator(np.random.PCG64(7))
    n = 4096
    pos = rng.uniform(-0.2, 1.2, (3, n)).astype(np.float32)
    vel = rng.normal(0.0, 2.0, (3, n)).astype(np.float32)
    vel[0, :8] = [np.nan, np.inf, -np.inf, 1e38, -1e38, 0.0, -0.0, np.nan]
    vel[1, 8:12] = np.inf
    p = [pos[k].copy() for k in range(3)]
    v = [vel[k].copy() for k in range(3)]
    ref.apply_ops(OPS, 0.01, p, v)
    return pos, vel, np.stack(p), np.stack(v)


def main():
    if not ref.available():
        raise SystemExit("oracle/_ref/libref.so missing: run `make -C oracle ref` with a reference checkout")
    data = {}
    for name, c in cases().items():
        r = run_case(c)
        data[f"{name}/pos"] = c["pos"]
        data[f"{name}/vel"] = c["vel"]
        data[f"{name}/meta"] = np.array([c["cs"], *c["dims"], c["mass"]], np.float64)
        data[f"{name}/grid_sha256"] = np.array(digest(r["cell_idx"], r["sorted_idx"], r["cell_start"]))
        for k in ("density", "pressure_accel", "viscosity_vel"):
            data[f"{name}/{k}"] = r[k]
    pos, vel, po, vo = epilogue_case()
    data["epilogue/pos"], data["epilogue/vel"] = pos, vel
    data["epilogue/pos_out"], data["epilogue/vel_out"] = po, vo
    data["epilogue/dt"] = np.array(0.01, np.float32)
    np.savez_compressed(os.path.join(HERE, "ref_sph.npz"), **data)
    print("wrote", os.path.join(HERE, "ref_sph.npz"))


if __name__ == "__main__":
    main()
