"""bench.py's reference arm runs on the host (the reference's own kernels
built for the host where oracle/_ref/libref.so exists, else the oracle port
of the step): its JSON line carries the contract's keys, and it uses every
core of the affinity mask even under torchrun's OMP_NUM_THREADS=1."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "ref65k",
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT,
                       env=env)
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "SPH particle-steps/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["warmup"] == 3 and d["steps"] == 1
    cb = d["cpu_baseline"]
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref
    assert cb["value"] == d["value"] and cb["sample"] and cb["cpu"]
    assert cb["kind"] == ("reference" if ref.available() else "port")
    assert cb["cores"] == len(os.sched_getaffinity(0))
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "ref65k"
