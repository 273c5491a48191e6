"""numpy binding of the CPU oracle (oracle/_build/liborc.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg as the checker. The product never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(_HERE, "_build", "liborc.so")
_lib = None

_f = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")


class SphParams(ctypes.Structure):
    _fields_ = [("h", ctypes.c_float), ("mass", ctypes.c_float), ("gas_constant", ctypes.c_float),
                ("rest_density", ctypes.c_float), ("viscosity", ctypes.c_float)]


class StepOp(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("p", ctypes.c_float * 7)]


class StepParams(ctypes.Structure):
    _fields_ = [("dt", ctypes.c_float), ("gravity", ctypes.c_float * 3), ("box_min", ctypes.c_float * 3),
                ("box_max", ctypes.c_float * 3), ("restitution", ctypes.c_float), ("flags", ctypes.c_uint32),
                ("n_ops", ctypes.c_uint32), ("ops", StepOp * 8)]


def build() -> None:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        u64, u32, f32, i32, vp = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_float, ctypes.c_int, ctypes.c_void_p
        f3 = ctypes.POINTER(ctypes.c_float)
        L.orc_uniform_f32.argtypes = [u64, u64, f32, f32, _f]
        L.orc_normal_f32.argtypes = [u64, u64, f32, f32, _f]
        L.orc_uniform_u32.argtypes = [u64, u64, _u]
        L.orc_morton30.argtypes = [u64, u64, _u]
        L.orc_lattice.argtypes = [u32, u32, u32, f32, f3, _f, _f, _f]
        L.orc_blobs.argtypes = [u64, u64, u32, f32, f32, f32, _f, _f, _f]
        L.orc_xorshift32_keys.argtypes = [u32, u64, u32, _u]
        L.orc_cell_of.restype = u32
        L.orc_cell_of.argtypes = [f32, f32, f32, f3, f32, u32, u32, u32]
        L.orc_grid_build.argtypes = [vp, vp, vp, u32, u64, f3, f32, u32, u32, u32, _u, _u, _u]
        L.orc_sort_pairs.argtypes = [_u, _u, u64, u32, u32]
        L.orc_cell_bounds.argtypes = [_u, u64, u64, _u, _u]
        L.orc_query.restype = u64
        L.orc_query.argtypes = [vp, vp, vp, u32, _u, _u, f3, f32, u32, u32, u32, f32, f32, f32, f32, vp, u64]
        L.orc_density.argtypes = [ctypes.POINTER(SphParams), _f, _f, _f, u64, f32, u32, u32, u32, _u, _u, _f, i32]
        L.orc_force.argtypes = [ctypes.POINTER(SphParams), u32, _f, _f, _f, _f, _f, _f, _f, u64, f32, u32, u32, u32,
                                _u, _u, f32, _f, _f, _f, vp, vp, vp, i32]
        L.orc_step.argtypes = [ctypes.POINTER(SphParams), ctypes.POINTER(StepParams), _f, _f, _f, _f, _f, _f, vp,
                               u64, f32, u32, u32, u32, _u, i32]
        L.orc_density_at.argtypes = [ctypes.POINTER(SphParams), _f, _f, _f, f32, u32, u32, u32, _u, _u, _u, u64,
                                     _f, i32]
        L.orc_force_at.argtypes = [ctypes.POINTER(SphParams), u32, _f, _f, _f, _f, _f, _f, _f, f32, u32, u32, u32,
                                   _u, _u, _u, u64, f32, _f, _f, _f, vp, vp, vp, i32]
        L.orc_apply_ops.argtypes = [ctypes.POINTER(StepParams), _f, _f, _f, _f, _f, _f, u64]
        L.orc_max_threads.restype = i32
        _lib = L
    return _lib


def _f3(v):
    return None if v is None else (ctypes.c_float * 3)(*v)


# ---- generators -----------------------------------------------------------
def uniform(seed, n, lo=0.0, hi=1.0):
    out = np.empty(n, np.float32)
    lib().orc_uniform_f32(seed, n, lo, hi, out)
    return out


def normal(seed, n, mean=0.0, sigma=1.0):
    out = np.empty(n, np.float32)
    lib().orc_normal_f32(seed, n, mean, sigma, out)
    return out


def uniform_u32(seed, n):
    out = np.empty(n, np.uint32)
    lib().orc_uniform_u32(seed, n, out)
    return out


def morton30(seed, n):
    out = np.empty(n, np.uint32)
    lib().orc_morton30(seed, n, out)
    return out


def xorshift32_keys(seed, n, mask):
    out = np.empty(n, np.uint32)
    lib().orc_xorshift32_keys(seed, n, mask, out)
    return out


def lattice(nx, ny, nz, spacing, lo=(0.0, 0.0, 0.0)):
    n = nx * ny * nz
    p = [np.empty(n, np.float32) for _ in range(3)]
    lib().orc_lattice(nx, ny, nz, spacing, _f3(lo), *p)
    return p


def blobs(seed, n, nblobs, clo, chi, sigma):
    p = [np.empty(n, np.float32) for _ in range(3)]
    lib().orc_blobs(seed, n, nblobs, clo, chi, sigma, *p)
    return p


# ---- grid -------------------------------------------------------------------
def cell_of(p, origin, cs, dims):
    return int(lib().orc_cell_of(p[0], p[1], p[2], _f3(origin), cs, *dims))


def grid_build(px, py, pz, cs, dims, origin=None):
    """SoA positions -> (cell_idx, sorted_idx, cell_start)."""
    n = px.size
    C = dims[0] * dims[1] * dims[2]
    ci, si, cst = np.empty(n, np.uint32), np.empty(n, np.uint32), np.empty(C + 1, np.uint32)
    px, py, pz = (np.ascontiguousarray(a, np.float32) for a in (px, py, pz))
    lib().orc_grid_build(px.ctypes.data, py.ctypes.data, pz.ctypes.data, 1, n, _f3(origin), cs, *dims, ci, si, cst)
    return ci, si, cst


def grid_build_aos(xyz, cs, dims, origin=None):
    xyz = np.ascontiguousarray(xyz, np.float32)
    n = xyz.shape[0]
    C = dims[0] * dims[1] * dims[2]
    ci, si, cst = np.empty(n, np.uint32), np.empty(n, np.uint32), np.empty(C + 1, np.uint32)
    a = xyz.ctypes.data
    lib().orc_grid_build(a, a + 4, a + 8, 3, n, _f3(origin), cs, *dims, ci, si, cst)
    return ci, si, cst


def sort_pairs(keys, vals, begin_bit=0, end_bit=32):
    k, v = np.array(keys, np.uint32), np.array(vals, np.uint32)
    lib().orc_sort_pairs(k, v, k.size, begin_bit, end_bit)
    return k, v


def cell_bounds(ids, num_cells):
    ids = np.ascontiguousarray(ids, np.uint32)
    s, e = np.empty(num_cells, np.uint32), np.empty(num_cells, np.uint32)
    lib().orc_cell_bounds(ids, ids.size, num_cells, s, e)
    return s, e


def query(px, py, pz, cell_start, sorted_idx, cs, dims, q, radius, origin=None):
    px, py, pz = (np.ascontiguousarray(a, np.float32) for a in (px, py, pz))
    L = lib()
    args = (px.ctypes.data, py.ctypes.data, pz.ctypes.data, 1, cell_start, sorted_idx, _f3(origin), cs, *dims,
            float(q[0]), float(q[1]), float(q[2]), radius)
    cnt = L.orc_query(*args, None, 0)
    hits = np.empty(max(cnt, 1), np.uint32)
    L.orc_query(*args, hits.ctypes.data, cnt)
    return hits[:cnt]


# ---- SPH ----------------------------------------------------------------------
def density(p: SphParams, px, py, pz, cs, dims, cell_start, sorted_idx, threads=1):
    out = np.empty(px.size, np.float32)
    lib().orc_density(ctypes.byref(p), px, py, pz, px.size, cs, *dims, cell_start, sorted_idx, out, threads)
    return out


def force(p: SphParams, terms, px, py, pz, vx, vy, vz, rho, cs, dims, cell_start, sorted_idx, dt, threads=1):
    n = px.size
    vo = [np.empty(n, np.float32) for _ in range(3)]
    ac = [np.empty(n, np.float32) for _ in range(3)]
    lib().orc_force(ctypes.byref(p), terms, px, py, pz, vx, vy, vz, rho, n, cs, *dims, cell_start, sorted_idx, dt,
                    *vo, *(a.ctypes.data for a in ac), threads)
    return vo, ac


def density_at(p: SphParams, px, py, pz, cs, dims, cell_start, sorted_idx, idx, threads=1):
    """Densities of particles idx only (all particles as neighbours)."""
    idx = np.ascontiguousarray(idx, np.uint32)
    out = np.empty(idx.size, np.float32)
    lib().orc_density_at(ctypes.byref(p), px, py, pz, cs, *dims, cell_start, sorted_idx, idx, idx.size, out,
                         threads)
    return out


def force_at(p: SphParams, terms, px, py, pz, vx, vy, vz, rho, cs, dims, cell_start, sorted_idx, idx, dt,
             threads=1):
    """(velocities, accelerations) of particles idx only."""
    idx = np.ascontiguousarray(idx, np.uint32)
    m = idx.size
    vo = [np.empty(m, np.float32) for _ in range(3)]
    ac = [np.empty(m, np.float32) for _ in range(3)]
    lib().orc_force_at(ctypes.byref(p), terms, px, py, pz, vx, vy, vz, rho, cs, *dims, cell_start, sorted_idx, idx,
                       m, dt, *vo, *(a.ctypes.data for a in ac), threads)
    return vo, ac


def step(p: SphParams, sp: StepParams, pos, vel, cs, dims, threads=1, want_density=False):
    """One manifest step in place on lists of numpy arrays pos, vel."""
    n = pos[0].size
    C = dims[0] * dims[1] * dims[2]
    work = np.empty(4 * n + C + 1, np.uint32)
    rho = np.empty(n, np.float32) if want_density else None
    lib().orc_step(ctypes.byref(p), ctypes.byref(sp), *pos, *vel, None if rho is None else rho.ctypes.data, n, cs,
                   *dims, work, threads)
    return rho


def apply_ops(sp: StepParams, pos, vel) -> None:
    """sp.ops[0..n_ops) in order on every particle, in place (orc_apply_ops)."""
    lib().orc_apply_ops(ctypes.byref(sp), *pos, *vel, pos[0].size)


def max_threads():
    return lib().orc_max_threads()
