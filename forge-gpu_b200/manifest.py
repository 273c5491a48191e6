"""TOML simulation manifests -> FieldSet + Pipeline -> a captured run.

The host side of the reference's `forge run` for particle simulations:
  * schema   -- SimManifest and its defaults (forge-manifest/src/schema.rs:6-225);
  * validate -- the manifest checks (validate.rs:17-81);
  * initial_fields -- field initialisation (manifest_runner.rs:192-318), with
    a seeded generator where the reference draws from an unseeded
    thread_rng (:274), so runs are reproducible;
  * build_pipeline -- forces -> integrate -> constraints, with the
    density + pressure + viscosity fusion (manifest_runner.rs:320-544);
  * run_manifest -- warm-up substeps, one CUDA graph of `substeps` steps,
    replays (manifest_runner.rs:11-105), and the summary lines of
    `forge run` (bin/forge.rs:176-190).
A fused pipeline (SphFused followed by per-particle modules) is one
forge_sph_step per substep, so the captured graph holds one grid build +
density + force/epilogue per substep. Springs and custom expression forces
are not particle-hot-path modules and are rejected.

    python manifest.py run examples/dam-break.toml [--seed S] [--device D]
"""
from __future__ import annotations

import argparse
import math
import sys
import time
import tomllib
from dataclasses import dataclass, field

import numpy as np

import forge_sph


class ManifestError(ValueError):
    """A manifest that does not parse, validate, or map onto the hot path."""


@dataclass
class SimResult:
    """SimResult (forge-manifest/src/lib.rs): final positions (count, 3)."""
    positions: np.ndarray
    count: int
    steps: int
    elapsed_secs: float
    pipeline: list = field(default_factory=list)

    @property
    def throughput(self) -> float:
        """particle-steps/s, as `forge run` prints it (bin/forge.rs:181-182)."""
        return self.count * self.steps / self.elapsed_secs if self.elapsed_secs > 0 else float("inf")


_SIM_DEFAULTS = {"type": "particles", "dt": 0.001, "substeps": 1, "duration": 1.0}   # schema.rs:38-41
_INIT_DEFAULTS = {"random": {"min": [-1.0, -1.0, -1.0], "max": [1.0, 1.0, 1.0]},       # schema.rs:82-85
                  "grid": {"spacing": 0.1, "origin": [0.0, 0.0, 0.0]}}
_FORCE_DEFAULTS = {"gravity": {"value": [0.0, -9.81, 0.0]}, "drag": {"coefficient": 0.01},  # schema.rs:126-128
                   "wind": {"direction": [], "strength": 1.0}}
_RESTITUTION = 0.5                                                                      # schema.rs:163


@dataclass
class Manifest:
    """SimManifest (schema.rs:6-20) as plain Python values, defaults applied."""
    simulation: dict
    fields: list
    forces: list
    constraints: list
    springs: dict | None
    spatial: dict | None

    @classmethod
    def from_toml(cls, text: str) -> "Manifest":
        try:
            raw = tomllib.loads(text)
        except tomllib.TOMLDecodeError as e:
            raise ManifestError(f"TOML parse error: {e}") from None
        if "simulation" not in raw or "name" not in raw["simulation"]:
            raise ManifestError("TOML parse error: missing [simulation] name")
        sim = dict(_SIM_DEFAULTS, **raw["simulation"])
        fields = []
        for f in raw.get("fields", []):
            f = dict({"type": "vec3f"}, **f)
            init = f.get("init")
            if init is not None:
                kind = init.get("type")
                if kind not in ("zero", "random", "constant", "grid"):
                    raise ManifestError(f"TOML parse error: unknown init type {kind!r} for field {f['name']!r}")
                if kind == "constant" and "value" not in init:
                    raise ManifestError(f"TOML parse error: constant init of {f['name']!r} needs a value")
                f["init"] = dict(_INIT_DEFAULTS.get(kind, {}), **init)
            fields.append(f)
        forces = []
        for f in raw.get("forces", []):
            kind = f.get("type")
            required = {"sph_density": ("smoothing_radius",), "sph_pressure": ("gas_constant", "rest_density"),
                        "sph_viscosity": ("coefficient",), "custom": ("expr",)}
            if kind not in ("gravity", "drag", "wind") and kind not in required:
                raise ManifestError(f"TOML parse error: unknown force type {kind!r}")
            for key in required.get(kind, ()):
                if key not in f:
                    raise ManifestError(f"TOML parse error: force {kind!r} needs {key!r}")
            forces.append(dict(_FORCE_DEFAULTS.get(kind, {}), **f))
        constraints = []
        for c in raw.get("constraints", []):
            kind = c.get("type")
            if kind not in ("ground_plane", "sphere", "box"):
                raise ManifestError(f"TOML parse error: unknown constraint type {kind!r}")
            need = {"sphere": ("center", "radius"), "box": ("min", "max")}.get(kind, ())
            for key in need:
                if key not in c:
                    raise ManifestError(f"TOML parse error: constraint {kind!r} needs {key!r}")
            defaults = {"restitution": _RESTITUTION, **({"y": 0.0} if kind == "ground_plane" else {})}
            constraints.append(dict(defaults, **c))
        spatial = raw.get("spatial")
        if spatial is not None:
            if "cell_size" not in spatial:
                raise ManifestError("TOML parse error: [spatial] needs cell_size")
            spatial = dict({"type": "hashgrid", "grid_dims": [32, 32, 32]}, **spatial)
        return cls(sim, fields, forces, constraints, raw.get("springs"), spatial)

    @classmethod
    def from_file(cls, path: str) -> "Manifest":
        try:
            with open(path, encoding="utf-8") as fh:
                text = fh.read()
        except OSError as e:
            raise ManifestError(f"Failed to read '{path}': {e}") from None
        return cls.from_toml(text)

    def particle_count(self) -> int:
        """schema.rs:210-223: simulation.count, else the first field count, else 1000."""
        if self.simulation.get("count") is not None:
            return int(self.simulation["count"])
        for f in self.fields:
            if f.get("count") is not None:
                return int(f["count"])
        return 1000

    def total_steps(self) -> int:
        """Graph launches of the run: (duration / dt) / substeps, in f32 as the
        reference computes it (manifest_runner.rs:25)."""
        d = np.float32(self.simulation["duration"]) / np.float32(self.simulation["dt"])
        return int(d) // max(int(self.simulation["substeps"]), 1)


def validate(m: Manifest) -> list:
    """The reference's manifest checks (validate.rs:17-81): error messages."""
    errs = []
    sim = m.simulation
    if not sim.get("name"):
        errs.append("simulation.name is required")
    if sim["dt"] <= 0:
        errs.append(f"simulation.dt must be > 0, got {sim['dt']}")
    if sim["duration"] <= 0:
        errs.append(f"simulation.duration must be > 0, got {sim['duration']}")
    if sim["type"] == "particles" and m.particle_count() == 0:
        errs.append("particle simulation needs count > 0")
    for i, f in enumerate(m.forces):
        if f["type"] == "gravity" and len(f["value"]) != 3:
            errs.append(f"forces[{i}].gravity.value must have 3 components")
    for i, c in enumerate(m.constraints):
        if c["type"] == "sphere" and len(c["center"]) != 3:
            errs.append(f"constraints[{i}].sphere.center must have 3 components")
    return errs


def _vec3_init(n: int, init: dict | None, rng: np.random.Generator):
    """init_vec3 (manifest_runner.rs:268-310): three float32 arrays."""
    if init is None or init["type"] == "zero":
        return [np.zeros(n, np.float32) for _ in range(3)]
    if init["type"] == "random":
        mn = [float(v) for v in (list(init["min"]) + [-1.0] * 3)[:3]]
        mx = [float(v) for v in (list(init["max"]) + [1.0] * 3)[:3]]
        return [rng.uniform(np.float32(mn[k]), np.float32(mx[k]), n).astype(np.float32) for k in range(3)]
    if init["type"] == "constant":
        v = (list(init["value"]) + [0.0] * 3)[:3]
        return [np.full(n, np.float32(v[k]), np.float32) for k in range(3)]
    # grid: a horizontal X/Z sheet at height origin.y, side = ceil(sqrt(n)) (:291-308)
    sp = np.float32(init["spacing"])
    o = [np.float32(v) for v in (list(init["origin"]) + [0.0] * 3)[:3]]
    side = int(math.ceil(math.sqrt(n)))
    i = np.arange(n)
    return [(o[0] + (i % side).astype(np.float32) * sp).astype(np.float32), np.full(n, o[1], np.float32),
            (o[2] + (i // side).astype(np.float32) * sp).astype(np.float32)]


def initial_vec3(m: Manifest, seed: int = 0) -> dict:
    """The manifest's initial fields as the reference builds them on the host
    (init_vec3 / init_f32, manifest_runner.rs:192-310): base name -> (n, 3)
    Vec3f array for vec3f fields (position/velocity mapped to pos/vel), name
    -> (n,) array for f32 fields; zero pos/vel added when absent."""
    n = m.particle_count()
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for f in m.fields:
        base = {"position": "pos", "pos": "pos", "velocity": "vel", "vel": "vel"}.get(f["name"], f["name"])
        if f["type"] == "vec3f":
            out[base] = np.stack(_vec3_init(n, f.get("init"), rng), axis=1)
        elif f["type"] == "f32":
            init = f.get("init")
            v = float(init["value"][0]) if init is not None and init["type"] == "constant" else 0.0
            out[f["name"]] = np.full(n, np.float32(v), np.float32)
    for base in ("vel", "pos"):
        out.setdefault(base, np.zeros((n, 3), np.float32))
    return out


def initial_fields(m: Manifest, seed: int = 0) -> dict:
    """init_fields (manifest_runner.rs:192-234): name -> float32 array, vec3
    fields split into _x/_y/_z with position/velocity mapped to pos/vel;
    zero pos/vel added when absent."""
    n = m.particle_count()
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for f in m.fields:
        base = {"position": "pos", "pos": "pos", "velocity": "vel", "vel": "vel"}.get(f["name"], f["name"])
        if f["type"] == "vec3f":
            for a, arr in zip("xyz", _vec3_init(n, f.get("init"), rng)):
                out[f"{base}_{a}"] = arr
        elif f["type"] == "f32":
            init = f.get("init")
            v = float(init["value"][0]) if init is not None and init["type"] == "constant" else 0.0
            out[f["name"]] = np.full(n, np.float32(v), np.float32)
    for base in ("vel", "pos"):
        if f"{base}_x" not in out:
            for a in "xyz":
                out[f"{base}_{a}"] = np.zeros(n, np.float32)
    return out


def _grid_of(m: Manifest, default_cell: float):
    sp = m.spatial
    cell = float(sp["cell_size"]) if sp is not None else default_cell
    dims = tuple(int(v) for v in (list(sp["grid_dims"]) if sp is not None else []) + [32, 32, 32])[:3]
    return cell, dims


def _mass(rho0: float, n: int) -> float:
    """Particle mass rho0 / n * 0.001 in f32, as the reference computes it."""
    return float(np.float32(rho0) / np.float32(n) * np.float32(0.001))


def build_pipeline(m: Manifest) -> forge_sph.Pipeline:
    """build_pipeline (manifest_runner.rs:320-544): forces, integrate,
    constraints. With all three SPH forces present they become one
    SphFusedModule (mass = rest_density / n * 0.001, :370); the forces are
    otherwise added one by one (sph_density mass 1000 / n * 0.001, :437).
    Wind is ignored, as in the reference."""
    n = m.particle_count()
    kinds = [f["type"] for f in m.forces]
    if "custom" in kinds:
        raise ManifestError("custom expression forces are not on the particle hot path (no expression compiler)")
    if m.springs is not None:
        raise ManifestError("springs are not on the particle hot path")
    p = forge_sph.Pipeline()
    dens = next((f for f in m.forces if f["type"] == "sph_density"), None)
    pres = next((f for f in m.forces if f["type"] == "sph_pressure"), None)
    visc = next((f for f in m.forces if f["type"] == "sph_viscosity"), None)
    h = float(dens["smoothing_radius"]) if dens is not None else 0.025

    def vec(v, d):
        return [float(x) for x in (list(v) + list(d))[:3]]

    def simple(f):
        if f["type"] == "gravity":
            g = vec(f["value"], [0.0, -9.81, 0.0])
            p.add(forge_sph.GravityModule(*g))
        elif f["type"] == "drag":
            p.add(forge_sph.DragModule(float(f["coefficient"])))

    if dens is not None and pres is not None and visc is not None:
        cell, dims = _grid_of(m, h * 2.0)
        rho0 = float(pres["rest_density"])
        p.add(forge_sph.SphFusedModule(h, cell, dims, _mass(rho0, n), float(pres["gas_constant"]), rho0,
                                       float(visc["coefficient"])))
        for f in m.forces:
            simple(f)
    else:
        for f in m.forces:
            if f["type"] == "sph_density":
                cell, dims = _grid_of(m, h * 2.0)
                p.add(forge_sph.SphDensityModule(h, cell, dims, _mass(1000.0, n)))
            elif f["type"] == "sph_pressure":
                rho0 = float(f["rest_density"])
                p.add(forge_sph.SphPressureModule(h, _mass(rho0, n), float(f["gas_constant"]), rho0))
            elif f["type"] == "sph_viscosity":
                p.add(forge_sph.SphViscosityModule(h, _mass(1000.0, n), float(f["coefficient"])))
            else:
                simple(f)
    p.add(forge_sph.IntegrateModule())
    for c in m.constraints:
        e = float(c["restitution"])
        if c["type"] == "ground_plane":
            p.add(forge_sph.GroundPlaneModule(float(c["y"]), e))
        elif c["type"] == "sphere":
            p.add(forge_sph.SphereColliderModule(*vec(c["center"], [0.0] * 3), float(c["radius"]), e))
        else:
            lo, hi = vec(c["min"], [0.0] * 3), vec(c["max"], [1.0] * 3)
            p.add(forge_sph.BoxColliderModule(*lo, *hi, e))
    return p


def run_manifest(m: Manifest, device: int = 0, seed: int = 0, capture: bool = True,
                 steps: int | None = None) -> SimResult:
    """run_manifest (manifest_runner.rs:11-105): warm-up substeps, one CUDA
    graph of `substeps` pipeline steps on a side stream, replayed for the
    remaining steps (`steps` overrides the manifest's launch count). A
    pipeline that does not fuse runs eagerly (its torch modules synchronise)."""
    import torch
    errs = validate(m)
    if errs:
        raise ManifestError("; ".join(errs))
    if not torch.cuda.is_available():
        raise ManifestError("No GPU")
    n = m.particle_count()
    dt = float(np.float32(m.simulation["dt"]))
    sub = max(int(m.simulation["substeps"]), 1)
    total = m.total_steps() if steps is None else int(steps)
    fields = forge_sph.FieldSet(n, device)
    for name, arr in initial_vec3(m, seed).items():  # uploaded and split into SoA on the GPU
        if arr.ndim == 2:
            fields.add_vec3(name, arr)
        else:
            fields.add_f32(name, arr)
    pipe = build_pipeline(m)
    fused = pipe._fused_plan() is not None
    with torch.cuda.device(device):
        t0 = time.perf_counter()
        count = 0
        for _ in range(sub):  # warm-up: allocates the grid and the density field
            pipe.step(fields, dt)
            count += 1
        if total > 1:
            if capture and fused:
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=side):
                    for _ in range(sub):
                        pipe.step_async(fields, dt)
                for _ in range(1, total):
                    graph.replay()
                    count += sub
            else:
                for _ in range(1, total):
                    for _ in range(sub):
                        pipe.step_async(fields, dt)
                    count += sub
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        grid = fields.u32_fields.get("_grid")
        if grid is not None:
            grid.check()
    pos = fields.positions()  # interleaved on the GPU, one copy back
    return SimResult(pos, n, count, elapsed, [mod.name() for mod in pipe.modules])


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="manifest.py", description="Run a particle simulation manifest")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("manifest")
    r.add_argument("--seed", type=int, default=0)
    r.add_argument("--device", type=int, default=0)
    r.add_argument("--steps", type=int, default=None, help="graph launches (default: duration / dt / substeps)")
    a = ap.parse_args(argv)
    try:
        m = Manifest.from_file(a.manifest)
        pipe = build_pipeline(m)
        fused = pipe._fused_plan() is not None
        print(f"  Pipeline: {len(pipe)} modules ({', '.join(x.name() for x in pipe.modules)})"
              + ("; fused into one forge_sph_step per substep" if fused else ""))
        res = run_manifest(m, a.device, a.seed, steps=a.steps)
    except (ManifestError, forge_sph.ForgeError) as e:
        print(f"Simulation failed: {e}", file=sys.stderr)
        return 1
    print("Simulation complete")
    print(f"  Steps: {res.steps}")
    print(f"  Time: {res.elapsed_secs:.3f}s")
    print(f"  Throughput: {res.throughput:.2e} particle-steps/s")
    print("\n  Sample final positions:")
    for i in range(min(5, res.count)):
        x, y, z = res.positions[i]
        print(f"    #{i}: ({x:.3f}, {y:.3f}, {z:.3f})")
    return 0


if __name__ == "__main__":
    sys.exit(main())
