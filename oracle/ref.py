"""numpy binding of oracle/_ref/libref.so: the reference's own SPH kernel
strings built for the host (see ref_extract.py, ref_shim.h, ref_driver.cpp).

TEST INFRASTRUCTURE ONLY: used to make and re-check the golden fixtures in
tests/golden/ and, where it was built, as the timed reference arm of bench.py.
The product never imports it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(_HERE, "_ref", "libref.so")
_lib = None
_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")


def available() -> bool:
    return os.path.exists(LIB)


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB)
        f32, i32 = ctypes.c_float, ctypes.c_int
        f3 = ctypes.POINTER(ctypes.c_float)
        L.ref_grid_build.argtypes = [_f, _f, _f, f32, i32, i32, i32, i32, _u, _u, _u]
        L.ref_density.argtypes = [_f, _f, _f, _f, _u, _u, f32, f32, f32, i32, i32, i32, i32, i32]
        L.ref_pressure_jacobi.argtypes = [_f, _f, _f, _f, _f, _f, _f, _u, _u, f32, f32, f32, f32, f32, i32, i32, i32,
                                          f32, i32, _f, _f, _f]
        L.ref_viscosity_jacobi.argtypes = [_f, _f, _f, _f, _f, _f, _f, _u, _u, f32, f32, f32, f32, i32, i32, i32, f32,
                                           i32, _f, _f, _f]
        L.ref_gravity.argtypes = [_f, _f, _f, f32, f32, f32, f32, i32, i32]
        L.ref_integrate.argtypes = [_f, _f, _f, _f, _f, _f, f32, i32, i32]
        L.ref_box_collider.argtypes = [_f, _f, _f, _f, _f, _f, f3, f3, f32, i32, i32]
        L.ref_drag.argtypes = [_f, _f, _f, f32, f32, i32, i32]
        L.ref_ground.argtypes = [_f, _f, f32, f32, i32, i32]
        L.ref_sphere_collide.argtypes = [_f, _f, _f, _f, _f, _f, f32, f32, f32, f32, f32, i32, i32]
        L.ref_manifest_step.argtypes = [_f, _f, _f, _f, _f, _f, _f, _u, _u, _u, f32, f32, f32, f32, f32, f32, i32,
                                        i32, i32, f32, f3, f3, f3, f32, i32, i32]
        _lib = L
    return _lib


def _f3(v):
    return (ctypes.c_float * 3)(*v)


def grid_build(pos, cs, dims):
    n = pos[0].size
    C = dims[0] * dims[1] * dims[2]
    ci, cst, si = np.empty(n, np.uint32), np.empty(C + 1, np.uint32), np.empty(n, np.uint32)
    lib().ref_grid_build(*pos, cs, *dims, n, ci, cst, si)
    return ci, si, cst


def density(pos, cell_start, sorted_idx, h, mass, cs, dims, threads=1):
    out = np.empty(pos[0].size, np.float32)
    lib().ref_density(*pos, out, cell_start, sorted_idx, h, mass, cs, *dims, pos[0].size, threads)
    return out


def pressure(pos, vel, rho, cell_start, sorted_idx, h, mass, k, rho0, cs, dims, dt):
    """sph_pressure in Jacobi form: velocities after the kernel, every
    particle against the unmodified input velocities."""
    vel = [np.array(v, np.float32) for v in vel]
    out = [np.empty_like(v) for v in vel]
    lib().ref_pressure_jacobi(*pos, *vel, rho, cell_start, sorted_idx, h, mass, k, rho0, cs, *dims, dt,
                              pos[0].size, *out)
    return out


def viscosity(pos, vel, rho, cell_start, sorted_idx, h, mass, mu, cs, dims, dt):
    vel = [np.array(v, np.float32) for v in vel]
    out = [np.empty_like(v) for v in vel]
    lib().ref_viscosity_jacobi(*pos, *vel, rho, cell_start, sorted_idx, h, mass, mu, cs, *dims, dt, pos[0].size,
                               *out)
    return out


def apply_ops(ops, dt, pos, vel, threads=1):
    """Per-particle modules in list order, in place. ops: (kind, params)
    with the kinds of forge_sph.h's FORGE_OP_* (1 gravity, 2 drag,
    3 integrate, 4 ground plane, 5 sphere collider, 6 box collider)."""
    L, n = lib(), pos[0].size
    for kind, p in ops:
        if kind == 1:
            L.ref_gravity(*vel, p[0], p[1], p[2], dt, n, threads)
        elif kind == 2:
            L.ref_drag(*vel, p[0], dt, n, threads)
        elif kind == 3:
            L.ref_integrate(*pos, *vel, dt, n, threads)
        elif kind == 4:
            L.ref_ground(pos[1], vel[1], p[0], p[1], n, threads)
        elif kind == 5:
            L.ref_sphere_collide(*pos, *vel, p[0], p[1], p[2], p[3], p[4], n, threads)
        elif kind == 6:
            L.ref_box_collider(*pos, *vel, _f3(p[0:3]), _f3(p[3:6]), p[6], n, threads)
        else:
            raise ValueError(kind)


class ManifestStep:
    """The reference's unfused manifest step (in place, threads in parallel,
    the reference's own in-place velocity race included) -- the timed CPU
    reference arm."""

    def __init__(self, cfg, n):
        C = cfg.dims[0] * cfg.dims[1] * cfg.dims[2]
        self.cfg, self.n = cfg, n
        self.rho = np.empty(n, np.float32)
        self.ci, self.si = np.empty(n, np.uint32), np.empty(n, np.uint32)
        self.cst = np.empty(C + 1, np.uint32)

    def __call__(self, pos, vel, threads):
        c = self.cfg
        lib().ref_manifest_step(*pos, *vel, self.rho, self.ci, self.cst, self.si, c.h, c.mass, c.gas_constant,
                                c.rest_density, c.viscosity, c.cell_size, *c.dims, c.dt, _f3(c.gravity),
                                _f3(c.box_min), _f3(c.box_max), c.restitution, self.n, threads)
