"""Shared helpers for the GPU parity tests (device <-> numpy, tolerances)."""
import numpy as np


def dev(torch, a, dtype=None):
    """numpy -> CUDA tensor (uint32 stored as int32 bit patterns)."""
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    t = torch.from_numpy(a.copy()).cuda()
    return t if dtype is None else t.to(dtype)


def host_u32(t):
    return t.cpu().numpy().view(np.uint32)


def host_f32(t):
    return t.cpu().numpy().astype(np.float32, copy=False)


def assert_force_close(a_gpu, a_cpu, scale, rel=1e-4, what="accel"):
    """|a_gpu - a_cpu| <= rel * sum_j |term_j| / rho_i per component (the
    norm-wise criterion: cancellation in the sum cannot inflate the error)."""
    for k in range(3):
        err = np.abs(a_gpu[k].astype(np.float64) - a_cpu[k])
        tol = rel * scale[k].astype(np.float64) + 1e-30
        bad = np.nonzero(err > tol)[0]
        assert bad.size == 0, (f"{what}[{k}]: {bad.size} particles off, worst i={bad[np.argmax(err[bad] / tol[bad])]}"
                               f" err={err[bad].max():.3e} tol={tol[bad].min():.3e}")
