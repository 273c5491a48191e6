"""GPU parity: Onesweep radix sort and find_cell_boundaries through the C ABI,
bit-exact against the oracle / the reference's known answers."""
import json
import os

import numpy as np
import pytest

import forge_sph
import oracle
import workloads
from _util import dev, host_u32

pytestmark = pytest.mark.gpu
GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def test_radix_small_kat(cuda):
    # tests/radix_sort_test.rs:14-48
    k = GOLD["radix_small"]
    keys = dev(cuda, np.array(k["keys"], np.uint32))
    vals = dev(cuda, np.arange(16, dtype=np.uint32))
    s = forge_sph.RadixSorter(16, 0)
    s.sort(keys, vals, 16, 4)
    s.check()
    assert host_u32(keys).tolist() == k["sorted_keys"]
    assert host_u32(vals).tolist() == k["sorted_vals"]


@pytest.mark.parametrize("name", ["radix_medium", "radix_cpu_ref"])
def test_radix_xorshift_kats(cuda, name):
    # tests/radix_sort_test.rs:50-136
    k = GOLD[name]
    keys_np = oracle.xorshift32_keys(k["seed"], k["n"], k["mask"])
    keys, vals = dev(cuda, keys_np), dev(cuda, np.arange(k["n"], dtype=np.uint32))
    s = forge_sph.RadixSorter(k["n"], 0)
    s.sort(keys, vals, k["n"], k["num_bits"])
    s.check()
    assert host_u32(keys).tolist() == k["sorted_keys"]
    assert host_u32(vals).tolist() == k["sorted_vals"]


def test_sort_argument_checks(cuda):
    s = forge_sph.RadixSorter(100, 0)
    k = cuda.zeros(200, dtype=cuda.int32, device="cuda")
    with pytest.raises(forge_sph.ForgeError):
        s.sort(k, k.clone(), 200, 8)  # n > max_n (radix_sort.rs:86)
    with pytest.raises(forge_sph.ForgeError):
        s.sort(k, k.clone(), 50, 6)  # num_bits % 4 != 0 (radix_sort.rs:87)
    with pytest.raises(forge_sph.ForgeError) as e:
        s.sort_pairs(k, k.clone(), 50, 4, 4)
    assert e.value.code == forge_sph.FORGE_ERR_INVALID_ARG


# tile edges of the small (1024-key) and large (4096-key) tiles
SIZES = [0, 1, 2, 31, 4095, 4096, 4097, 8191, 8192, 8193, 65537, 131_072, 131_073, 1_000_003]
RANGES = [(0, 32), (0, 16), (4, 20), (8, 30), (0, 1), (0, 8), (28, 32)]


@pytest.mark.parametrize("n", SIZES)
def test_sort_pairs_uniform_vs_oracle(cuda, n):
    rng = np.random.default_rng(n + 7)
    keys_np = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    vals_np = rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
    s = forge_sph.RadixSorter(max(n, 1), 0)
    for lo, hi in RANGES:
        keys, vals = dev(cuda, keys_np), dev(cuda, vals_np)
        s.sort_pairs(keys, vals, n, lo, hi)
        s.check()
        ek, ev = oracle.sort_pairs(keys_np, vals_np, lo, hi)
        assert np.array_equal(host_u32(keys)[:n], ek), (n, lo, hi)
        assert np.array_equal(host_u32(vals)[:n], ev), (n, lo, hi)


@pytest.mark.parametrize("kind", ["dups4", "allsame", "sorted", "reversed", "morton"])
@pytest.mark.parametrize("n", [100_000, 300_000])
def test_sort_pairs_skewed_keys(cuda, kind, n):
    rng = np.random.default_rng(11)
    if kind == "dups4":
        keys_np = rng.integers(0, 4, n).astype(np.uint32)
    elif kind == "allsame":
        keys_np = np.full(n, 0xDEADBEEF, np.uint32)
    elif kind == "sorted":
        keys_np = np.sort(rng.integers(0, 2 ** 32, n, dtype=np.uint64)).astype(np.uint32)
    elif kind == "reversed":
        keys_np = np.sort(rng.integers(0, 2 ** 32, n, dtype=np.uint64))[::-1].astype(np.uint32)
    else:
        keys_np = workloads.sort_keys("morton", n, seed=3)
    vals_np = np.arange(n, dtype=np.uint32)
    s = forge_sph.RadixSorter(n, 0)
    keys, vals = dev(cuda, keys_np), dev(cuda, vals_np)
    s.sort_pairs(keys, vals, n, 0, 32 if kind != "morton" else 30)
    s.check()
    ek, ev = oracle.sort_pairs(keys_np, vals_np, 0, 32 if kind != "morton" else 30)
    assert np.array_equal(host_u32(keys), ek)
    assert np.array_equal(host_u32(vals), ev)


def test_caller_alt_buffers_swap_semantics(cuda):
    n = 50_000
    keys_np = workloads.sort_keys("uniform", n, seed=5)
    s = forge_sph.RadixSorter(n, 0)
    for lo, hi in ((0, 8), (0, 16), (0, 24), (0, 32)):
        keys, vals = dev(cuda, keys_np), dev(cuda, np.arange(n, dtype=np.uint32))
        ka, va = cuda.empty_like(keys), cuda.empty_like(vals)
        in_alt = s.sort_pairs(keys, vals, n, lo, hi, keys_alt=ka, vals_alt=va)
        passes = (hi - lo + 7) // 8
        assert in_alt == (passes % 2 == 1)
        rk, rv = (ka, va) if in_alt else (keys, vals)
        ek, ev = oracle.sort_pairs(keys_np, np.arange(n, dtype=np.uint32), lo, hi)
        assert np.array_equal(host_u32(rk), ek) and np.array_equal(host_u32(rv), ev)


@pytest.mark.parametrize("kind", ["uniform", "morton"])
def test_sort_full_size_cfg1_properties(cuda, kind):
    """cfg1 at full size (2^28 pairs): sortedness, stability (values are the
    input positions, so equal keys must keep increasing values) and the
    permutation property keys_out == keys_in[vals_out]."""
    torch = cuda
    n = 1 << 28
    bits = 32 if kind == "uniform" else 30
    keys_np = workloads.sort_keys(kind, n)
    keys_in = dev(torch, keys_np)
    del keys_np
    keys = keys_in.clone()
    vals = torch.arange(n, dtype=torch.int32, device="cuda")
    s = forge_sph.RadixSorter(n, 0)
    s.sort_pairs(keys, vals, n, 0, bits)
    s.check()
    k64 = keys.to(torch.int64) & 0xFFFFFFFF
    assert bool((k64[1:] >= k64[:-1]).all())
    eq = k64[1:] == k64[:-1]
    assert bool((vals[1:][eq] > vals[:-1][eq]).all())
    assert bool((keys_in[vals.long()] == keys).all())
    assert int(vals.to(torch.int64).sum()) == n * (n - 1) // 2


def test_cell_bounds_kat(cuda):
    k = GOLD["cell_bounds"]
    ids = dev(cuda, np.array(k["sorted"], np.uint32))
    start = cuda.zeros(8, dtype=cuda.int32, device="cuda")
    end = cuda.zeros(8, dtype=cuda.int32, device="cuda")
    forge_sph.find_cell_boundaries(ids, start, end, 8, k["num_cells"], 0)
    assert host_u32(start).tolist() == k["start"]
    assert host_u32(end).tolist() == k["end"]


@pytest.mark.parametrize("n,C", [(0, 10), (1, 1), (1, 5000), (10_000, 64_000), (200_000, 4096), (5, 1_000_000)])
def test_cell_bounds_vs_oracle(cuda, n, C):
    rng = np.random.default_rng(n + C)
    ids_np = np.sort(rng.integers(0, C, n)).astype(np.uint32)
    start = cuda.full((C,), 7, dtype=cuda.int32, device="cuda")
    end = cuda.full((C,), 7, dtype=cuda.int32, device="cuda")
    forge_sph.find_cell_boundaries(dev(cuda, ids_np) if n else start[:0], start, end, n, C, 0)
    es, ee = oracle.cell_bounds(ids_np, C)
    assert np.array_equal(host_u32(start), es)
    assert np.array_equal(host_u32(end), ee)


def test_lookback_wait_gives_up_and_is_reported(cuda):
    """Failure detection without a GPU fault: the test hook makes the first
    pass skip tile id 0, so tile 1's decoupled look-back waits on a status
    word nothing writes. The wait is bounded (4096 polls here): the kernel
    records the timeout and returns, forge_sorter_check reports
    FORGE_ERR_TIMEOUT, and the same sorter then sorts correctly again."""
    n = 5 * 4096 + 17
    keys_np = oracle.uniform_u32(7, n)
    s = forge_sph.RadixSorter(n, 0)
    L = forge_sph.lib()
    keys, vals = dev(cuda, keys_np), dev(cuda, np.arange(n, dtype=np.uint32))
    forge_sph.check(L.forge_sorter_set_test_fault(s._h, 1, 1 << 12))
    s.sort_pairs(keys, vals, n, 0, 32)
    with pytest.raises(forge_sph.ForgeError, match="look-back"):
        s.check()
    forge_sph.check(L.forge_sorter_set_test_fault(s._h, 0, 0))
    keys, vals = dev(cuda, keys_np), dev(cuda, np.arange(n, dtype=np.uint32))
    s.sort_pairs(keys, vals, n, 0, 32)
    s.check()
    ek, ev = oracle.sort_pairs(keys_np, np.arange(n, dtype=np.uint32))
    assert np.array_equal(host_u32(keys), ek) and np.array_equal(host_u32(vals), ev)
