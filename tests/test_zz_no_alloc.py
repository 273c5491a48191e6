"""GPU test of forge_sort_pairs_static, the sort entry point that allocates
nothing (for callers that cannot call cudaMalloc: fixed device-memory
budgets, plug-in hosts that own the allocator, latency-critical loops that
cannot take an allocation's implicit synchronisation). Its scratch lives in a
fixed array inside the library, shared by every call.

It must give exactly the handle-based sorter's result (integer work:
tolerance zero), including on a second call right after the first, which
reuses the same scratch. This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest

import forge_sph
import workloads

pytestmark = pytest.mark.gpu


def _static_sort(torch, keys, vals, lo, hi):
    L = forge_sph.lib()
    rc = L.forge_sort_pairs_static(keys.data_ptr(), vals.data_ptr(), keys.numel(), lo, hi,
                                   torch.cuda.current_stream().cuda_stream)
    forge_sph.check(rc)


@pytest.mark.parametrize("n,lo,hi", [(300_000, 0, 32), (forge_sph.STATIC_SORT_MAX_N, 0, 24)])
def test_static_sort_matches_handle_sorter_twice(cuda, n, lo, hi):
    torch = cuda
    sorter = forge_sph.RadixSorter(n, 0)
    for call, seed in enumerate((11, 12)):  # two calls in a row on the shared scratch
        keys_np = workloads.sort_keys("uniform", n, seed=seed + n)
        if call == 1:
            keys_np &= np.uint32(0xFFF0FFFF)  # different digit statistics on the second call
        k_ref = torch.from_numpy(keys_np.view(np.int32).copy()).cuda()
        v_ref = torch.arange(n, dtype=torch.int32, device="cuda")
        k_st, v_st = k_ref.clone(), v_ref.clone()
        sorter.sort_pairs(k_ref, v_ref, n, lo, hi)
        sorter.check()
        _static_sort(torch, k_st, v_st, lo, hi)
        torch.cuda.synchronize()
        assert torch.equal(k_st, k_ref), f"call {call}: keys differ"
        assert torch.equal(v_st, v_ref), f"call {call}: values differ"


def test_static_sort_rejects_oversize_and_accepts_empty(cuda):
    torch = cuda
    L = forge_sph.lib()
    n = forge_sph.STATIC_SORT_MAX_N + 1
    k = torch.zeros(n, dtype=torch.int32, device="cuda")
    rc = L.forge_sort_pairs_static(k.data_ptr(), k.data_ptr(), n, 0, 32, None)
    assert rc == forge_sph.FORGE_ERR_CAPACITY
    assert "static maximum" in forge_sph.last_error()
    assert L.forge_sort_pairs_static(None, None, 0, 0, 32, None) == forge_sph.FORGE_OK
