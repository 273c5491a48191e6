"""Python host side of the B200 particle hot path, over the C ABI of
libforge_sph.so (include/forge_sph.h).

Mirrors the reference's Rust interface for this path (paths relative to the
forge-gpu project root) so callers and tests read like the reference's own:

  RadixSorter(max_n, ordinal).sort(keys, values, n, num_bits)
        forge-runtime/src/radix_sort.rs:26-220 (same swap-by-ownership result)
  find_cell_boundaries(sorted_ids, cell_start, cell_end, n, num_cells, ordinal)
        forge-runtime/src/radix_sort.rs:229-317
  HashGrid(cell_size, grid_dims, origin, max_particles, device)
        .build(positions) / .position_to_cell(p) / .query_neighbors(p, r, positions)
        forge-runtime/src/hashgrid.rs:21-193
  FieldSet, Pipeline, SphFusedModule, SphDensityModule, SphPressureModule,
  SphViscosityModule, GravityModule, IntegrateModule, BoxColliderModule
        forge-manifest/src/modules/mod.rs:12-117, modules/builtins/*.rs

Device buffers are torch CUDA tensors (the role of the reference's
Array<T>): torch is plumbing only, every computation runs in the library's
sm_100a kernels. There is no CPU fallback: if the shared library is missing
or no GPU is present, calls raise ForgeError.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FORGE_SPH_LIB") or os.path.join(_HERE, "libforge_sph.so")

FORGE_OK = 0
FORGE_ERR_INVALID_ARG = -1
FORGE_ERR_CAPACITY = -2
FORGE_ERR_CUDA = -3
FORGE_ERR_TIMEOUT = -4
FORGE_ERR_NCCL = -5
FORGE_ERR_DEVICE = -6

OP_GRAVITY, OP_DRAG, OP_INTEGRATE, OP_GROUND, OP_SPHERE, OP_BOX = 1, 2, 3, 4, 5, 6
# neighbour-pass kernel families (forge_grid_set_walk)
WALK_AUTO, WALK_THREAD, WALK_GROUP4, WALK_GROUP8, WALK_GROUP16, WALK_ROWS, WALK_TILE = 0, 1, 2, 3, 4, 5, 6
STEP_MAX_OPS = 8

TERM_PRESSURE = 1
TERM_VISCOSITY = 2
STEP_GRAVITY = 1
STEP_INTEGRATE = 2
STEP_BOX = 4

_CODE_NAMES = {
    FORGE_ERR_INVALID_ARG: "InvalidArgument",
    FORGE_ERR_CAPACITY: "Capacity",
    FORGE_ERR_CUDA: "Cuda",
    FORGE_ERR_TIMEOUT: "Timeout",
    FORGE_ERR_NCCL: "Nccl",
    FORGE_ERR_DEVICE: "Device",
}

# Every symbol include/forge_sph.h declares.
EXPORTED = (
    "forge_last_error", "forge_abi_version",
    "forge_sorter_create", "forge_sorter_sort_pairs", "forge_sorter_check", "forge_sorter_destroy",
    "forge_sorter_set_test_fault",
    "forge_cell_bounds",
    "forge_grid_create", "forge_grid_build", "forge_grid_build_aos", "forge_grid_query",
    "forge_grid_check", "forge_grid_destroy",
    "forge_sph_density", "forge_sph_force", "forge_sph_step",
    "forge_grid_profile_enable", "forge_grid_profile_read", "forge_grid_set_x_window", "forge_grid_set_walk",
    "forge_io_create", "forge_io_destroy", "forge_io_upload", "forge_io_download", "forge_io_upload_vec3",
    "forge_io_download_vec3",
    "forge_sort_pairs_static",
    "forge_sph_force_step",
    "forge_slab_create", "forge_slab_destroy", "forge_slab_classify", "forge_slab_compact", "forge_slab_x_hist",
    "forge_nccl_unique_id", "forge_slab_comm_create", "forge_slab_comm_destroy", "forge_slab_exchange",
    "forge_apply_ops", "forge_slab_exchange_rho", "forge_slab_comm_set_bounds", "forge_slab_comm_set_timeout", "forge_sph_force_step_zone", "forge_slab_exchange_begin", "forge_slab_exchange_end",
)
ZONE_BOUNDARY, ZONE_INTERIOR, ZONE_PREPARE = 1, 2, 3
STATIC_SORT_MAX_N = 1 << 20


class ForgeError(RuntimeError):
    """Error returned by the library (mirrors ForgeError, forge-runtime/src/error.rs:7-22)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{_CODE_NAMES.get(code, code)}: {message}")
        self.code = code


class SphParams(ctypes.Structure):
    _fields_ = [("h", ctypes.c_float), ("mass", ctypes.c_float), ("gas_constant", ctypes.c_float),
                ("rest_density", ctypes.c_float), ("viscosity", ctypes.c_float)]


class StepOp(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("p", ctypes.c_float * 7)]


class StepParams(ctypes.Structure):
    _fields_ = [("dt", ctypes.c_float), ("gravity", ctypes.c_float * 3), ("box_min", ctypes.c_float * 3),
                ("box_max", ctypes.c_float * 3), ("restitution", ctypes.c_float), ("flags", ctypes.c_uint32),
                ("n_ops", ctypes.c_uint32), ("ops", StepOp * 8)]


class ForceZone(ctypes.Structure):
    """forge_force_zone: the x-split of forge_sph_force_step_zone."""
    _fields_ = [("mode", ctypes.c_uint32), ("inner_lo", ctypes.c_float), ("inner_hi", ctypes.c_float),
                ("guard_lo", ctypes.c_float), ("guard_hi", ctypes.c_float)]


_lib = None


def lib() -> ctypes.CDLL:
    """Load libforge_sph.so (built in-tree by `make -C forge-gpu_b200`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ForgeError(FORGE_ERR_CUDA, f"{LIB_PATH} is missing: build it with `make -C forge-gpu_b200`")
    L = ctypes.CDLL(LIB_PATH)
    vp, u64, u32, i32, f32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int, ctypes.c_float
    pvp = ctypes.POINTER(ctypes.c_void_p)
    sig = {
        "forge_last_error": (u64, [ctypes.c_char_p, u64]),
        "forge_abi_version": (i32, []),
        "forge_sorter_create": (i32, [u64, i32, pvp]),
        "forge_sorter_sort_pairs": (i32, [vp, vp, vp, vp, vp, u64, u32, u32, ctypes.POINTER(i32), vp]),
        "forge_sorter_check": (i32, [vp, vp]),
        "forge_sorter_destroy": (None, [vp]),
        "forge_sorter_set_test_fault": (i32, [vp, u32, u32]),
        "forge_cell_bounds": (i32, [vp, vp, vp, u64, u64, vp]),
        "forge_grid_create": (i32, [f32, u32, u32, u32, ctypes.POINTER(f32), u64, i32, pvp]),
        "forge_grid_build": (i32, [vp, vp, vp, vp, u64, vp, vp, vp, vp]),
        "forge_grid_build_aos": (i32, [vp, vp, u64, vp, vp, vp, vp]),
        "forge_grid_query": (i32, [vp, vp, vp, vp, vp, vp, vp, u64, f32, vp, vp, vp, u64, vp]),
        "forge_grid_check": (i32, [vp, vp]),
        "forge_grid_destroy": (None, [vp]),
        "forge_sph_density": (i32, [vp, ctypes.POINTER(SphParams), vp, vp, vp, u64, vp, vp]),
        "forge_sph_force": (i32, [vp, ctypes.POINTER(SphParams), u32, vp, vp, vp, vp, vp, vp, vp, u64, f32,
                                  vp, vp, vp, vp, vp, vp, vp]),
        "forge_sph_step": (i32, [vp, ctypes.POINTER(SphParams), ctypes.POINTER(StepParams), vp, vp, vp, vp, vp,
                                 vp, vp, u64, vp]),
        "forge_grid_profile_enable": (i32, [vp, u32]),
        "forge_grid_set_x_window": (i32, [vp, u32, u32]),
        "forge_grid_set_walk": (i32, [vp, i32]),
        "forge_io_create": (i32, [u64, i32, pvp]),
        "forge_io_destroy": (None, [vp]),
        "forge_io_upload": (i32, [vp, pvp, pvp, u32, u64, vp]),
        "forge_io_download": (i32, [vp, pvp, pvp, u32, u64, vp]),
        "forge_io_upload_vec3": (i32, [vp, vp, vp, vp, vp, u64, vp]),
        "forge_io_download_vec3": (i32, [vp, vp, vp, vp, vp, u64, vp]),
        "forge_sort_pairs_static": (i32, [vp, vp, u64, u32, u32, vp]),
        "forge_nccl_unique_id": (i32, [ctypes.c_char_p]),
        "forge_slab_comm_create": (i32, [ctypes.c_char_p, i32, i32, i32, u64, f32, f32, f32, pvp]),
        "forge_slab_comm_destroy": (None, [vp]),
        "forge_slab_comm_set_bounds": (i32, [vp, f32, f32]),
        "forge_apply_ops": (i32, [ctypes.POINTER(StepParams), vp, vp, vp, vp, vp, vp, u64, i32, vp]),
        "forge_slab_comm_set_timeout": (i32, [vp, ctypes.c_double]),
        "forge_slab_exchange": (i32, [vp, vp, u64, u64, i32, ctypes.POINTER(u64), ctypes.POINTER(u64), vp]),
        "forge_slab_exchange_rho": (i32, [vp, vp, vp]),
        "forge_slab_create": (i32, [u64, i32, pvp]),
        "forge_slab_destroy": (None, [vp]),
        "forge_slab_classify": (i32, [vp, vp, u64, f32, f32, f32, u32, vp, vp, vp]),
        "forge_slab_compact": (i32, [vp, u64, u32, u64, vp, u64, vp]),
        "forge_slab_x_hist": (i32, [vp, vp, vp, u64, f32, f32, u32, vp, vp]),
        "forge_sph_force_step": (i32, [vp, ctypes.POINTER(SphParams), ctypes.POINTER(StepParams), vp, vp, vp, vp,
                                       vp, vp, vp, u64, u64, vp]),
        "forge_sph_force_step_zone": (i32, [vp, ctypes.POINTER(SphParams), ctypes.POINTER(StepParams), vp, vp, vp,
                                            vp, vp, vp, vp, u64, u64, ctypes.POINTER(ForceZone), vp]),
        "forge_slab_exchange_begin": (i32, [vp, vp, u64, u64, vp]),
        "forge_slab_exchange_end": (i32, [vp, vp, u64, ctypes.POINTER(u64), ctypes.POINTER(u64), vp]),
        "forge_grid_profile_read": (i32, [vp, ctypes.POINTER(f32), u32, ctypes.POINTER(u32)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().forge_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != FORGE_OK:
        raise ForgeError(rc, last_error())


def ptr(t) -> int | None:
    """Device address of a torch tensor (None for None)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ForgeError(FORGE_ERR_INVALID_ARG, "expected a CUDA tensor")
    if not t.is_contiguous():
        raise ForgeError(FORGE_ERR_INVALID_ARG, "expected a contiguous tensor")
    return t.data_ptr()


def _stream(stream=None) -> int | None:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise ForgeError(FORGE_ERR_CUDA, "no CUDA device: the particle hot path has no CPU fallback")
    return torch


# ---------------------------------------------------------------------------
# Radix sort
# ---------------------------------------------------------------------------
class RadixSorter:
    """RadixSorter (radix_sort.rs:26-220): pre-allocated stable key/value sorter."""

    def __init__(self, max_n: int, ordinal: int = 0):
        _torch()
        h = ctypes.c_void_p()
        check(lib().forge_sorter_create(max_n, ordinal, ctypes.byref(h)))
        self._h = h
        self.max_n = max_n
        self.ordinal = ordinal

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.forge_sorter_destroy(h)
            self._h = None

    def sort_pairs(self, keys, vals, n=None, begin_bit=0, end_bit=32, keys_alt=None, vals_alt=None,
                   stream=None) -> bool:
        """Raw C-ABI sort. Returns True if the result is in keys_alt/vals_alt."""
        n = keys.numel() if n is None else n
        where = ctypes.c_int(0)
        check(lib().forge_sorter_sort_pairs(self._h, ptr(keys), ptr(vals), ptr(keys_alt), ptr(vals_alt), n,
                                            begin_bit, end_bit, ctypes.byref(where), _stream(stream)))
        return bool(where.value)

    def sort(self, keys, values, n: int, num_bits: int) -> None:
        """RadixSorter::sort (radix_sort.rs:79-220): sorts the low num_bits
        bits; keys/values hold the result afterwards. Asserts n <= max_n and
        num_bits % 4 == 0, <= 32, as the reference does (:86-87)."""
        if n > self.max_n:
            raise ForgeError(FORGE_ERR_CAPACITY, f"n={n} exceeds max_n={self.max_n}")
        if num_bits % 4 != 0 or num_bits > 32:
            raise ForgeError(FORGE_ERR_INVALID_ARG, "num_bits must be multiple of 4, <= 32")
        if n == 0 or num_bits == 0:
            return
        self.sort_pairs(keys, values, n, 0, num_bits)

    def check(self, stream=None) -> None:
        check(lib().forge_sorter_check(self._h, _stream(stream)))


def find_cell_boundaries(sorted_cell_ids, cell_start, cell_end, n: int, num_cells: int, ordinal: int = 0,
                         stream=None) -> None:
    """find_cell_boundaries (radix_sort.rs:229-317)."""
    torch = _torch()
    with torch.cuda.device(ordinal):
        check(lib().forge_cell_bounds(ptr(sorted_cell_ids), ptr(cell_start), ptr(cell_end), n, num_cells,
                                      _stream(stream)))


# ---------------------------------------------------------------------------
# Hash grid
# ---------------------------------------------------------------------------
class HashGrid:
    """HashGrid (hashgrid.rs:21-193) with a GPU build and a GPU batched query."""

    def __init__(self, cell_size: float, grid_dims, origin=(0.0, 0.0, 0.0), max_particles: int = 0,
                 device: int = 0):
        torch = _torch()
        self.cell_size = float(cell_size)
        self.dim_x, self.dim_y, self.dim_z = (int(d) for d in grid_dims)
        self.origin = tuple(float(o) for o in origin)
        self.max_particles = int(max_particles)
        self.device = device
        o = (ctypes.c_float * 3)(*self.origin)
        h = ctypes.c_void_p()
        check(lib().forge_grid_create(self.cell_size, self.dim_x, self.dim_y, self.dim_z, o, self.max_particles,
                                      device, ctypes.byref(h)))
        self._h = h
        dev = torch.device("cuda", device)
        C = self.num_cells()
        self.cell_start = torch.zeros(C + 1, dtype=torch.int32, device=dev)
        self.sorted_indices = torch.zeros(max(self.max_particles, 1), dtype=torch.int32, device=dev)
        self.cell_indices = torch.zeros(max(self.max_particles, 1), dtype=torch.int32, device=dev)
        self.num_particles = 0
        self._positions = None

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.forge_grid_destroy(h)
            self._h = None

    @property
    def handle(self):
        return self._h

    def set_walk(self, walk: int) -> None:
        """Neighbour-pass kernel family (WALK_*; WALK_AUTO by particle count)."""
        check(lib().forge_grid_set_walk(self._h, walk))

    def set_x_window(self, cx0: int, nxw: int) -> None:
        """Index only global cells [cx0, cx0 + nxw) along x (a shard's slab);
        every particle built must lie inside (forge_grid_set_x_window)."""
        check(lib().forge_grid_set_x_window(self._h, int(cx0), int(nxw)))

    def num_cells(self) -> int:
        return self.dim_x * self.dim_y * self.dim_z

    def build(self, positions, stream=None) -> None:
        """HashGrid::build (hashgrid.rs:82-125). positions: (n,3) float32
        tensor (Vec3f AoS) on the grid's device, or a tuple (px, py, pz)."""
        torch = _torch()
        if isinstance(positions, (tuple, list)):
            px, py, pz = positions
            n = px.numel()
            check(lib().forge_grid_build(self._h, ptr(px), ptr(py), ptr(pz), n, ptr(self.cell_indices),
                                         ptr(self.sorted_indices), ptr(self.cell_start), _stream(stream)))
            self._positions = (px, py, pz)
        else:
            if not torch.is_tensor(positions) or positions.dim() != 2 or positions.shape[1] != 3:
                raise ForgeError(FORGE_ERR_INVALID_ARG, "positions must be an (n, 3) float32 tensor")
            n = positions.shape[0]
            xyz = positions.to(device=torch.device("cuda", self.device), dtype=torch.float32).contiguous()
            check(lib().forge_grid_build_aos(self._h, ptr(xyz), n, ptr(self.cell_indices),
                                             ptr(self.sorted_indices), ptr(self.cell_start), _stream(stream)))
            self._positions = (xyz[:, 0].contiguous(), xyz[:, 1].contiguous(), xyz[:, 2].contiguous())
        self.num_particles = n

    def position_to_cell(self, pos) -> int:
        """HashGrid::position_to_cell (hashgrid.rs:128-139), host arithmetic in f32."""
        import numpy as np
        cs = np.float32(self.cell_size)
        c = []
        for a, o, d in zip(pos, self.origin, (self.dim_x, self.dim_y, self.dim_z)):
            v = np.floor((np.float32(a) - np.float32(o)) / cs)
            iv = 0 if np.isnan(v) else int(max(min(v, 2 ** 31 - 1), -(2 ** 31)))
            c.append(min(max(iv, 0), d - 1))
        return c[0] + c[1] * self.dim_x + c[2] * self.dim_x * self.dim_y

    def query_batch(self, qx, qy, qz, radius: float, stream=None):
        """Batched GPU query: returns (counts, offsets, hits) CUDA tensors."""
        torch = _torch()
        if self._positions is None:
            raise ForgeError(FORGE_ERR_INVALID_ARG, "grid has not been built")
        px, py, pz = self._positions
        nq = qx.numel()
        dev = qx.device
        counts = torch.empty(max(nq, 1), dtype=torch.int32, device=dev)
        offsets = torch.empty(nq + 1, dtype=torch.int32, device=dev)
        L, st = lib(), _stream(stream)
        check(L.forge_grid_query(self._h, ptr(px), ptr(py), ptr(pz), ptr(qx), ptr(qy), ptr(qz), nq, radius,
                                 ptr(counts), ptr(offsets), None, 0, st))
        total = int(offsets[nq].item()) if nq else 0
        hits = torch.empty(max(total, 1), dtype=torch.int32, device=dev)
        check(L.forge_grid_query(self._h, ptr(px), ptr(py), ptr(pz), ptr(qx), ptr(qy), ptr(qz), nq, radius,
                                 ptr(counts), ptr(offsets), ptr(hits), total, st))
        check(L.forge_grid_check(self._h, st))
        return counts[:nq], offsets, hits[:total]

    def query_neighbors(self, pos, radius: float, positions=None):
        """HashGrid::query_neighbors (hashgrid.rs:145-193): indices within
        radius of pos, in the reference's walk order (a Python list)."""
        torch = _torch()
        dev = torch.device("cuda", self.device)
        q = [torch.tensor([float(v)], dtype=torch.float32, device=dev) for v in pos]
        _, _, hits = self.query_batch(q[0], q[1], q[2], radius)
        return [int(v) for v in hits.cpu().tolist()]

    def check(self, stream=None) -> None:
        check(lib().forge_grid_check(self._h, _stream(stream)))


# ---------------------------------------------------------------------------
# Field I/O (manifest_runner.rs:192-269, :83-92)
# ---------------------------------------------------------------------------
def _host_ptrs(arrays):
    """Host addresses of float32 numpy arrays or (pinned) CPU tensors."""
    out = []
    for a in arrays:
        if hasattr(a, "data_ptr"):
            if a.is_cuda or a.dtype != _torch().float32 or not a.is_contiguous():
                raise ForgeError(FORGE_ERR_INVALID_ARG, "expected contiguous float32 host tensors")
            out.append(a.data_ptr())
        else:
            if a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"]:
                raise ForgeError(FORGE_ERR_INVALID_ARG, "expected contiguous float32 numpy arrays")
            out.append(a.ctypes.data)
    return out


class FieldIO:
    """forge_io: host <-> device moves of particle fields through a pinned
    staging buffer, with Vec3f AoS <-> SoA conversion on the GPU."""

    def __init__(self, max_n: int, device: int = 0):
        h = ctypes.c_void_p()
        check(lib().forge_io_create(int(max_n), device, ctypes.byref(h)))
        self._h, self.max_n, self.device = h, int(max_n), device

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.forge_io_destroy(h)
            self._h = None

    @staticmethod
    def _vp(ptrs):
        return (ctypes.c_void_p * max(len(ptrs), 1))(*ptrs)

    def upload(self, host, dev, stream=None) -> None:
        """host[k] (float32 numpy / CPU tensor) -> dev[k] (CUDA tensor), asynchronous."""
        n = len(dev[0]) if dev else 0
        check(lib().forge_io_upload(self._h, self._vp(_host_ptrs(host)), self._vp([ptr(d) for d in dev]), len(dev),
                                    n, _stream(stream)))

    def download(self, dev, host, stream=None) -> None:
        """dev[k] -> host[k]: enqueued on `stream` when every host array is
        pinned (synchronise before reading them), else returns when the data
        are on the host."""
        n = len(dev[0]) if dev else 0
        check(lib().forge_io_download(self._h, self._vp([ptr(d) for d in dev]), self._vp(_host_ptrs(host)),
                                      len(dev), n, _stream(stream)))

    def upload_vec3(self, xyz, x, y, z, stream=None) -> None:
        """(n, 3) float32 host array -> x, y, z CUDA columns."""
        (hp,) = _host_ptrs([xyz])
        check(lib().forge_io_upload_vec3(self._h, hp, ptr(x), ptr(y), ptr(z), len(x), _stream(stream)))

    def download_vec3(self, x, y, z, stream=None) -> np.ndarray:
        """x, y, z CUDA columns -> new (n, 3) float32 numpy array."""
        out = np.empty((len(x), 3), np.float32)
        check(lib().forge_io_download_vec3(self._h, ptr(x), ptr(y), ptr(z), out.ctypes.data, len(x),
                                           _stream(stream)))
        return out


# ---------------------------------------------------------------------------
# Manifest modules (forge-manifest/src/modules)
# ---------------------------------------------------------------------------
class FieldSet:
    """FieldSet (modules/mod.rs:12-66): named device arrays, SoA particles
    (pos_x..vel_z, manifest_runner.rs:205-213)."""

    def __init__(self, particle_count: int, device: int = 0):
        self.particle_count = particle_count
        self.device = device
        self.f32_fields: dict = {}
        self.u32_fields: dict = {}
        self._io = None

    def io(self) -> FieldIO:
        if self._io is None:
            self._io = FieldIO(max(self.particle_count, 1), self.device)
        return self._io

    def add_f32(self, name: str, data) -> None:
        """Field `name` from host data (Array::from_vec): uploaded through
        the field I/O handle."""
        torch = _torch()
        a = np.ascontiguousarray(np.asarray(data, dtype=np.float32))
        t = torch.empty(a.shape, dtype=torch.float32, device=torch.device("cuda", self.device))
        if a.size:
            self.io().upload([a.reshape(-1)], [t.view(-1)])
        self.f32_fields[name] = t

    def add_vec3(self, base: str, xyz) -> None:
        """Fields base_x/_y/_z from an (n, 3) Vec3f array, split on the GPU
        (init_fields, manifest_runner.rs:205-213)."""
        torch = _torch()
        a = np.ascontiguousarray(np.asarray(xyz, dtype=np.float32).reshape(-1, 3))
        cols = [torch.empty(a.shape[0], dtype=torch.float32, device=torch.device("cuda", self.device))
                for _ in range(3)]
        if a.shape[0]:
            self.io().upload_vec3(a, *cols)
        for c, t in zip("xyz", cols):
            self.f32_fields[f"{base}_{c}"] = t

    def positions(self) -> np.ndarray:
        """pos_x/y/z interleaved into an (n, 3) array (the SimResult gather,
        manifest_runner.rs:83-92)."""
        f = self.f32_fields
        return self.io().download_vec3(f["pos_x"], f["pos_y"], f["pos_z"])

    def add_f32_zeros(self, name: str, n: int) -> None:
        torch = _torch()
        self.f32_fields[name] = torch.zeros(n, dtype=torch.float32, device=torch.device("cuda", self.device))

    def get_f32(self, name: str):
        return self.f32_fields.get(name)


class SimModule:
    """SimModule (modules/mod.rs:69-72)."""

    def name(self) -> str:
        raise NotImplementedError

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        raise NotImplementedError


class _SphGridMixin:
    """Owns the device grid handle the SPH modules rebuild every step (the
    reference keeps its grid arrays in FieldSet.u32_fields, sph_fused.rs:44-74)."""

    def _grid(self, fields: FieldSet):
        g = getattr(self, "_g", None)
        if g is None or g.max_particles < fields.particle_count:
            g = HashGrid(self.cell_size, self.grid_dims, (0.0, 0.0, 0.0), fields.particle_count, fields.device)
            self._g = g
        fields.u32_fields["_grid"] = g
        return g

    def _params(self) -> SphParams:
        return SphParams(self.smoothing_radius, self.particle_mass, getattr(self, "gas_constant", 0.0),
                         getattr(self, "rest_density", 0.0), getattr(self, "viscosity_coefficient", 0.0))


@dataclass
class SphDensityModule(SimModule, _SphGridMixin):
    """SphDensityModule (sph_density.rs:16-21, execute :388-501)."""
    smoothing_radius: float
    cell_size: float
    grid_dims: tuple
    particle_mass: float

    def name(self) -> str:
        return "sph_density"

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        g = self._grid(fields)
        n = fields.particle_count
        if "density" not in fields.f32_fields:
            fields.add_f32_zeros("density", n)
        f = fields.f32_fields
        check(lib().forge_sph_density(g.handle, ctypes.byref(self._params()), ptr(f["pos_x"]), ptr(f["pos_y"]),
                                      ptr(f["pos_z"]), n, ptr(f["density"]), _stream(stream)))


class _SphForceModule(SimModule):
    TERMS = 3

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        g = fields.u32_fields.get("_grid")
        if g is None:
            raise ForgeError(FORGE_ERR_INVALID_ARG, f"{self.name()} needs a preceding sph_density module")
        f = fields.f32_fields
        n = fields.particle_count
        p = SphParams(self.smoothing_radius, self.particle_mass, getattr(self, "gas_constant", 0.0),
                      getattr(self, "rest_density", 0.0), getattr(self, "coefficient", 0.0))
        check(lib().forge_sph_force(g.handle, ctypes.byref(p), self.TERMS, ptr(f["pos_x"]), ptr(f["pos_y"]),
                                    ptr(f["pos_z"]), ptr(f["vel_x"]), ptr(f["vel_y"]), ptr(f["vel_z"]),
                                    ptr(f["density"]), n, dt, ptr(f["vel_x"]), ptr(f["vel_y"]), ptr(f["vel_z"]),
                                    None, None, None, _stream(stream)))


@dataclass
class SphPressureModule(_SphForceModule):
    """SphPressureModule (sph_pressure.rs:9-161)."""
    smoothing_radius: float
    particle_mass: float
    gas_constant: float
    rest_density: float
    TERMS = TERM_PRESSURE

    def name(self) -> str:
        return "sph_pressure"


@dataclass
class SphViscosityModule(_SphForceModule):
    """SphViscosityModule (sph_viscosity.rs:9-154); Jacobi velocities."""
    smoothing_radius: float
    particle_mass: float
    coefficient: float
    TERMS = TERM_VISCOSITY

    def name(self) -> str:
        return "sph_viscosity"


@dataclass
class SphFusedModule(SimModule, _SphGridMixin):
    """SphFusedModule (sph_fused.rs:14-22, execute :413-733): grid rebuild,
    density, fused pressure+viscosity (Jacobi)."""
    smoothing_radius: float
    cell_size: float
    grid_dims: tuple
    particle_mass: float
    gas_constant: float
    rest_density: float
    viscosity_coefficient: float

    def name(self) -> str:
        return "sph_fused"

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        g = self._grid(fields)
        n = fields.particle_count
        if "density" not in fields.f32_fields:
            fields.add_f32_zeros("density", n)
        f = fields.f32_fields
        p = self._params()
        L, st = lib(), _stream(stream)
        check(L.forge_sph_density(g.handle, ctypes.byref(p), ptr(f["pos_x"]), ptr(f["pos_y"]), ptr(f["pos_z"]), n,
                                  ptr(f["density"]), st))
        check(L.forge_sph_force(g.handle, ctypes.byref(p), 3, ptr(f["pos_x"]), ptr(f["pos_y"]), ptr(f["pos_z"]),
                                ptr(f["vel_x"]), ptr(f["vel_y"]), ptr(f["vel_z"]), ptr(f["density"]), n, dt,
                                ptr(f["vel_x"]), ptr(f["vel_y"]), ptr(f["vel_z"]), None, None, None, st))


@dataclass
class GravityModule(SimModule):
    """GravityModule (gravity.rs). Standalone it runs as a torch op; inside a
    Pipeline after SphFusedModule it is fused into the force kernel."""
    gx: float = 0.0
    gy: float = -9.81
    gz: float = 0.0

    def name(self) -> str:
        return "gravity"

    def op(self):
        return OP_GRAVITY, [self.gx, self.gy, self.gz]

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        f = fields.f32_fields
        f["vel_x"].add_(self.gx * dt)
        f["vel_y"].add_(self.gy * dt)
        f["vel_z"].add_(self.gz * dt)


@dataclass
class IntegrateModule(SimModule):
    """IntegrateModule (integrate.rs:16-31)."""

    def name(self) -> str:
        return "integrate"

    def op(self):
        return OP_INTEGRATE, []

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        torch = _torch()
        f = fields.f32_fields
        for a in "xyz":
            v = f["vel_" + a]
            v.copy_(torch.where(torch.isfinite(v), v, torch.zeros_like(v)))
            f["pos_" + a].add_(v * dt)


@dataclass
class BoxColliderModule(SimModule):
    """BoxColliderModule (box_collider.rs:6-86)."""
    min_x: float = 0.0
    min_y: float = 0.0
    min_z: float = 0.0
    max_x: float = 1.0
    max_y: float = 1.0
    max_z: float = 1.0
    restitution: float = 1.0

    def name(self) -> str:
        return "box_collider"

    def op(self):
        return OP_BOX, [self.min_x, self.min_y, self.min_z, self.max_x, self.max_y, self.max_z, self.restitution]

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        torch = _torch()
        f = fields.f32_fields
        for a, lo, hi in (("x", self.min_x, self.max_x), ("y", self.min_y, self.max_y), ("z", self.min_z, self.max_z)):
            p, v = f["pos_" + a], f["vel_" + a]
            below, above = p < lo, p > hi
            v.copy_(torch.where(below, v.abs() * self.restitution, v))
            p.clamp_(min=lo)
            above = p > hi
            v.copy_(torch.where(above, -v.abs() * self.restitution, v))
            p.clamp_(max=hi)


@dataclass
class DragModule(SimModule):
    """DragModule (drag.rs:5-20): v *= 1 - coefficient * dt."""
    coefficient: float = 0.0

    def name(self) -> str:
        return "drag"

    def op(self):
        return OP_DRAG, [self.coefficient]

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        torch = _torch()
        d = torch.tensor(1.0, dtype=torch.float32) - torch.tensor(self.coefficient, dtype=torch.float32) * \
            torch.tensor(dt, dtype=torch.float32)
        for a in "xyz":
            fields.f32_fields["vel_" + a].mul_(d.item())


@dataclass
class GroundPlaneModule(SimModule):
    """GroundPlaneModule (ground_plane.rs:5-21): y < ground -> y = ground, vy = -vy * e."""
    y: float = 0.0
    restitution: float = 0.5

    def name(self) -> str:
        return "ground_plane"

    def op(self):
        return OP_GROUND, [self.y, self.restitution]

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        torch = _torch()
        py, vy = fields.f32_fields["pos_y"], fields.f32_fields["vel_y"]
        below = py < self.y
        vy.copy_(torch.where(below, -vy * self.restitution, vy))
        py.clamp_(min=self.y)


@dataclass
class SphereColliderModule(SimModule):
    """SphereColliderModule (sphere_collider.rs:5-41): push particles inside the
    sphere to its surface and reflect the inward normal velocity."""
    cx: float = 0.0
    cy: float = 0.0
    cz: float = 0.0
    radius: float = 1.0
    restitution: float = 0.5

    def name(self) -> str:
        return "sphere_collider"

    def op(self):
        return OP_SPHERE, [self.cx, self.cy, self.cz, self.radius, self.restitution]

    def execute(self, fields: FieldSet, dt: float, stream=None) -> None:
        torch = _torch()
        f = fields.f32_fields
        p = [f["pos_" + a] for a in "xyz"]
        v = [f["vel_" + a] for a in "xyz"]
        c = (self.cx, self.cy, self.cz)
        d = [p[k] - c[k] for k in range(3)]
        dist = torch.sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2])
        hit = (dist < self.radius) & (dist > 1e-8)
        inv = 1.0 / torch.where(hit, dist, torch.ones_like(dist))
        nrm = [d[k] * inv for k in range(3)]
        vn = v[0] * nrm[0] + v[1] * nrm[1] + v[2] * nrm[2]
        refl = hit & (vn < 0)
        for k in range(3):
            p[k].copy_(torch.where(hit, c[k] + nrm[k] * self.radius, p[k]))
            v[k].copy_(torch.where(refl, v[k] - (1 + self.restitution) * vn * nrm[k], v[k]))


class Pipeline:
    """Pipeline (modules/mod.rs:74-117). `step_async` recognises the manifest
    SPH pattern -- SphFusedModule followed only by per-particle modules
    (gravity, drag, integrate, ground plane, sphere and box colliders, in any
    order, at most 8) -- and runs it as ONE forge_sph_step call whose force
    kernel applies those modules in order; anything else runs module by
    module."""

    def __init__(self):
        self.modules: list = []

    def add(self, module: SimModule) -> None:
        self.modules.append(module)

    def __len__(self) -> int:
        return len(self.modules)

    def _fused_plan(self):
        if not self.modules or not isinstance(self.modules[0], SphFusedModule):
            return None
        rest = self.modules[1:]
        if len(rest) > STEP_MAX_OPS or not all(hasattr(m, "op") for m in rest):
            return None
        sp = StepParams()
        sp.n_ops = len(rest)
        for k, m in enumerate(rest):
            kind, params = m.op()
            sp.ops[k].kind = kind
            for q, v in enumerate(params):
                sp.ops[k].p[q] = v
        return sp

    def step_async(self, fields: FieldSet, dt: float, stream=None) -> None:
        sp = self._fused_plan()
        if sp is None:
            for m in self.modules:
                m.execute(fields, dt, stream)
            return
        sph = self.modules[0]
        g = sph._grid(fields)
        n = fields.particle_count
        if "density" not in fields.f32_fields:
            fields.add_f32_zeros("density", n)
        f = fields.f32_fields
        sp.dt = dt
        check(lib().forge_sph_step(g.handle, ctypes.byref(sph._params()), ctypes.byref(sp), ptr(f["pos_x"]),
                                   ptr(f["pos_y"]), ptr(f["pos_z"]), ptr(f["vel_x"]), ptr(f["vel_y"]),
                                   ptr(f["vel_z"]), ptr(f["density"]), n, _stream(stream)))

    def step(self, fields: FieldSet, dt: float, stream=None) -> None:
        torch = _torch()
        self.step_async(fields, dt, stream)
        (stream or torch.cuda.current_stream()).synchronize()

    def run(self, fields: FieldSet, dt: float, steps: int) -> None:
        for _ in range(steps):
            self.step(fields, dt)
