"""GPU test of the field I/O entry points (forge_io_*): SoA columns up and
down from pageable and pinned host memory, and Vec3f AoS <-> SoA through the
GPU, bit for bit (pure data movement); capacity and argument errors."""
import numpy as np
import pytest

import forge_sph

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 1000, 300_001])
@pytest.mark.parametrize("pinned", [False, True])
def test_soa_round_trip(cuda, n, pinned):
    rng = np.random.default_rng(n)
    host = [rng.standard_normal(n).astype(np.float32) for _ in range(6)]
    if pinned:
        host = [cuda.from_numpy(h).pin_memory() for h in host]
    dev = [cuda.empty(n, dtype=cuda.float32, device="cuda") for _ in range(6)]
    io = forge_sph.FieldIO(n, 0)
    io.upload(host, dev)
    want = [np.asarray(h) for h in host]
    for d, w in zip(dev, want):
        assert np.array_equal(d.cpu().numpy(), w)
    back = [np.empty(n, np.float32) for _ in range(6)]
    for d in dev:
        d.mul_(2.0)
    io.download(dev, back)
    for b, w in zip(back, want):
        assert np.array_equal(b, w * np.float32(2.0))


def test_vec3_aos_round_trip(cuda):
    n = 123_457
    xyz = np.random.default_rng(1).standard_normal((n, 3)).astype(np.float32)
    f = forge_sph.FieldSet(n, 0)
    f.add_vec3("pos", xyz)
    for k, c in enumerate("xyz"):
        assert np.array_equal(f.f32_fields["pos_" + c].cpu().numpy(), xyz[:, k])
    assert np.array_equal(f.positions(), xyz)


def test_capacity_and_bad_arguments(cuda):
    io = forge_sph.FieldIO(10, 0)
    dev = [cuda.empty(11, dtype=cuda.float32, device="cuda")]
    with pytest.raises(forge_sph.ForgeError, match="max_n"):
        io.upload([np.zeros(11, np.float32)], dev)
    with pytest.raises(forge_sph.ForgeError):
        io.upload([np.zeros(11, np.float64)], dev)
