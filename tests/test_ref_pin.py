"""Pins the oracle to the reference's OWN kernels (CPU, no GPU).

tests/golden/ref_sph.npz holds the outputs of the reference's kernel strings
(sph_density.rs:401-461, sph_pressure.rs:28-112, sph_viscosity.rs:27-106, its
GPU grid-build kernels sph_density.rs:72-122 and the per-particle modules),
built for the host and run by tests/golden/make_ref_fixtures.py. Both sides
round every float operation as written (no contraction), so the oracle must
reproduce them bit for bit. Where oracle/_ref/libref.so has been built here,
the fixtures are also regenerated and compared, so they cannot go stale.
"""
import hashlib
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden", "ref_sph.npz")
CASES = ("cube4k", "edges", "lowmass")
PHYS = dict(h=0.025, k=3.0, rho0=1000.0, mu=0.1)


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def case(gold, name):
    pos = [np.ascontiguousarray(gold[f"{name}/pos"][k]) for k in range(3)]
    vel = [np.ascontiguousarray(gold[f"{name}/vel"][k]) for k in range(3)]
    m = gold[f"{name}/meta"]
    cs, dims, mass = float(m[0]), tuple(int(x) for x in m[1:4]), float(m[4])
    return pos, vel, cs, dims, mass


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


@pytest.mark.parametrize("name", CASES)
def test_oracle_grid_is_the_reference_grid(gold, name):
    pos, _, cs, dims, _ = case(gold, name)
    ci, si, cst = oracle.grid_build(*pos, cs, dims)
    assert digest(ci, si, cst) == str(gold[f"{name}/grid_sha256"])


@pytest.mark.parametrize("name", CASES)
def test_oracle_density_bit_exact_vs_reference_kernel(gold, name):
    pos, _, cs, dims, mass = case(gold, name)
    _, si, cst = oracle.grid_build(*pos, cs, dims)
    p = oracle.SphParams(PHYS["h"], mass, PHYS["k"], PHYS["rho0"], PHYS["mu"])
    rho = oracle.density(p, *pos, cs, dims, cst, si)
    assert np.array_equal(rho.view(np.uint32), gold[f"{name}/density"].view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_oracle_pressure_and_viscosity_bit_exact_vs_reference_kernels(gold, name):
    pos, vel, cs, dims, mass = case(gold, name)
    _, si, cst = oracle.grid_build(*pos, cs, dims)
    p = oracle.SphParams(PHYS["h"], mass, PHYS["k"], PHYS["rho0"], PHYS["mu"])
    rho = gold[f"{name}/density"]
    zero = [np.zeros_like(v) for v in vel]
    vo, _ = oracle.force(p, 1, *pos, *zero, rho, cs, dims, cst, si, 1.0)
    assert np.array_equal(np.stack(vo).view(np.uint32), gold[f"{name}/pressure_accel"].view(np.uint32))
    vo, _ = oracle.force(p, 2, *pos, *vel, rho, cs, dims, cst, si, 1.0)
    assert np.array_equal(np.stack(vo).view(np.uint32), gold[f"{name}/viscosity_vel"].view(np.uint32))
    if name == "lowmass":  # the rho < 1e-6 rules really fire on both sides
        assert 0 < np.count_nonzero(rho < 1e-6) < rho.size


def test_oracle_modules_bit_exact_vs_reference_kernels(gold):
    from make_ref_fixtures import OPS
    pos = [np.ascontiguousarray(gold["epilogue/pos"][k]) for k in range(3)]
    vel = [np.ascontiguousarray(gold["epilogue/vel"][k]) for k in range(3)]
    sp = oracle.StepParams()
    sp.dt = float(gold["epilogue/dt"])
    sp.n_ops = len(OPS)
    for i, (kind, prm) in enumerate(OPS):
        sp.ops[i].kind = kind
        for j, x in enumerate(prm):
            sp.ops[i].p[j] = x
    oracle.apply_ops(sp, pos, vel)
    assert np.array_equal(np.stack(pos).view(np.uint32), gold["epilogue/pos_out"].view(np.uint32))
    assert np.array_equal(np.stack(vel).view(np.uint32), gold["epilogue/vel_out"].view(np.uint32))


def test_fixtures_regenerate_from_the_reference_build(gold):
    import ref
    if not ref.available():
        pytest.skip("oracle/_ref/libref.so not built (needs a reference checkout)")
    from make_ref_fixtures import cases, epilogue_case, run_case
    for name, c in cases().items():
        r = run_case(c)
        for k in ("density", "pressure_accel", "viscosity_vel"):
            assert np.array_equal(r[k].view(np.uint32), gold[f"{name}/{k}"].view(np.uint32)), (name, k)
        assert digest(r["cell_idx"], r["sorted_idx"], r["cell_start"]) == str(gold[f"{name}/grid_sha256"])
    _, _, po, vo = epilogue_case()
    assert np.array_equal(po.view(np.uint32), gold["epilogue/pos_out"].view(np.uint32))
    assert np.array_equal(vo.view(np.uint32), gold["epilogue/vel_out"].view(np.uint32))
