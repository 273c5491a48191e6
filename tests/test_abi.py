"""CPU tests: the C-ABI library loads, exports exactly what include/forge_sph.h
declares, and the host-side mirror's pure logic (no compute calls)."""
import ctypes
import os
import re

import pytest

import forge_sph

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "forge_sph.h")).read()
    return set(re.findall(r"^FORGE_API\s+[\w\s\*]+?\b(forge_\w+)\(", txt, flags=re.M))


def test_header_and_wrapper_agree():
    assert header_symbols() == set(forge_sph.EXPORTED)


def test_library_exports_every_declared_symbol():
    L = forge_sph.lib()
    for s in header_symbols():
        assert hasattr(L, s), s
    assert L.forge_abi_version() == 1


def test_error_paths_without_gpu():
    L = forge_sph.lib()
    h = ctypes.c_void_p()
    assert L.forge_sorter_create(1 << 30, 0, ctypes.byref(h)) == forge_sph.FORGE_ERR_INVALID_ARG
    assert "max_n" in forge_sph.last_error()
    assert L.forge_grid_create(0.0, 4, 4, 4, None, 16, 0, ctypes.byref(h)) == forge_sph.FORGE_ERR_INVALID_ARG
    assert L.forge_sorter_sort_pairs(None, None, None, None, None, 0, 0, 32, None, None) == \
        forge_sph.FORGE_ERR_INVALID_ARG
    assert L.forge_cell_bounds(None, None, None, 0, 0, None) == forge_sph.FORGE_OK


def test_pipeline_fused_plan():
    p = forge_sph.Pipeline()
    p.add(forge_sph.SphFusedModule(0.025, 0.025, (40, 40, 40), 1.0, 3.0, 1000.0, 0.1))
    p.add(forge_sph.GravityModule(0.0, -9.81, 0.0))
    p.add(forge_sph.DragModule(0.5))
    p.add(forge_sph.IntegrateModule())
    p.add(forge_sph.GroundPlaneModule(0.1, 0.3))
    p.add(forge_sph.SphereColliderModule(0.5, 0.5, 0.5, 0.2, 0.4))
    p.add(forge_sph.BoxColliderModule(0, 0, 0, 1, 1, 1, 0.5))
    sp = p._fused_plan()
    assert sp is not None and sp.n_ops == 6
    assert [sp.ops[k].kind for k in range(6)] == [forge_sph.OP_GRAVITY, forge_sph.OP_DRAG, forge_sph.OP_INTEGRATE,
                                                  forge_sph.OP_GROUND, forge_sph.OP_SPHERE, forge_sph.OP_BOX]
    assert list(sp.ops[0].p)[:3] == pytest.approx([0.0, -9.81, 0.0])
    assert sp.ops[5].p[6] == pytest.approx(0.5)
    q = forge_sph.Pipeline()
    q.add(forge_sph.GravityModule())
    assert q._fused_plan() is None  # no SPH module first
    r = forge_sph.Pipeline()
    r.add(forge_sph.SphFusedModule(0.025, 0.025, (40, 40, 40), 1.0, 3.0, 1000.0, 0.1))
    r.add(forge_sph.SphDensityModule(0.025, 0.025, (40, 40, 40), 1.0))
    assert r._fused_plan() is None  # a neighbour pass after it is not an epilogue op


def test_step_params_layout_matches_header():
    # dt, g[3], box min/max, restitution, flags, n_ops, 8 x (kind + 7 floats)
    assert ctypes.sizeof(forge_sph.StepParams) == 4 * (1 + 3 + 3 + 3 + 1 + 1 + 1 + 8 * 8)


def test_no_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(forge_sph.ForgeError):
        forge_sph.RadixSorter(16)


def test_sharded_entry_points_reject_bad_arguments_without_gpu():
    """The sharded-step entry points check their arguments before any device
    call (no GPU needed)."""
    L = forge_sph.lib()
    bad = forge_sph.FORGE_ERR_INVALID_ARG
    z = forge_sph.ForceZone(forge_sph.ZONE_BOUNDARY, 0.1, 0.9, 0.05, 0.95)
    sp, stp = forge_sph.SphParams(), forge_sph.StepParams()
    assert L.forge_sph_force_step_zone(None, ctypes.byref(sp), ctypes.byref(stp), *([None] * 7), 0, 0,
                                       ctypes.byref(z), None) == bad
    assert "NULL grid" in forge_sph.last_error()
    assert L.forge_slab_comm_set_timeout(None, 1.0) == bad
    assert L.forge_slab_comm_set_bounds(None, 0.0, 1.0) == bad
    assert L.forge_slab_exchange_begin(None, None, 0, 0, None) == bad
    n_own, ng = ctypes.c_uint64(), ctypes.c_uint64()
    assert L.forge_slab_exchange_end(None, None, 0, ctypes.byref(n_own), ctypes.byref(ng), None) == bad
    assert L.forge_slab_exchange_rho(None, None, None) == bad
    assert L.forge_slab_comm_create(None, 0, 1, 0, 16, 0.0, 1.0, 0.1, None) == bad


def header_defines(prefix):
    txt = open(os.path.join(ROOT, "include", "forge_sph.h")).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"^#define (" + prefix + r"\w+)\s+(\d+)u?\b", txt,
                                                                 flags=re.M)}


def test_walk_and_zone_constants_match_header():
    """The neighbour-pass families and force-zone modes the Python mirror and
    bench.py pass through the C ABI are the header's values."""
    import bench
    walks = header_defines("FORGE_WALK_")
    assert walks, "no FORGE_WALK_* in the header"
    for name, v in walks.items():
        assert getattr(forge_sph, name[len("FORGE_"):]) == v, name
    assert set(bench.WALKS.values()) == set(walks.values())
    zones = header_defines("FORGE_ZONE_")
    assert zones == {"FORGE_ZONE_BOUNDARY": 1, "FORGE_ZONE_INTERIOR": 2, "FORGE_ZONE_PREPARE": 3}
