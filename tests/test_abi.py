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
    p.add(forge_sph.IntegrateModule())
    p.add(forge_sph.BoxColliderModule(0, 0, 0, 1, 1, 1, 0.5))
    sp = p._fused_plan()
    assert sp is not None and sp.flags == 7
    assert list(sp.gravity) == pytest.approx([0.0, -9.81, 0.0])
    assert sp.restitution == pytest.approx(0.5)
    q = forge_sph.Pipeline()
    q.add(forge_sph.GravityModule())
    assert q._fused_plan() is None
    r = forge_sph.Pipeline()
    r.add(forge_sph.SphFusedModule(0.025, 0.025, (40, 40, 40), 1.0, 3.0, 1000.0, 0.1))
    r.add(forge_sph.IntegrateModule())
    r.add(forge_sph.GravityModule())  # gravity after integrate: not the fusable order
    assert r._fused_plan() is None


def test_no_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(forge_sph.ForgeError):
        forge_sph.RadixSorter(16)
