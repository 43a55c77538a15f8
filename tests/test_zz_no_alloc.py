"""Allocation-free GEMM entry point (mllm_gemm_q4_noalloc) against the allocating one (mllm_gemm_q4).

Some callers of this library cannot call cudaMalloc — a host runtime that owns all device memory
through its own pool, or a latency-sensitive thread that cannot afford cudaMalloc's implicit device
synchronisation.  mllm_gemm_q4_noalloc serves them from a fixed scratch array inside the library.
This file is collected last so that a failure here does not hide the results of the other tests."""
import ctypes

import numpy as np
import pytest

from conftest import pkg


def _case(rng, rows, cols, m):
    P = pkg()
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    packed, sc = P.quant_q4(w)
    x = rng.standard_normal((m, cols), dtype=np.float32)
    return packed, sc, x


@pytest.mark.gpu
def test_noalloc_gemm_matches_allocating_entry_on_two_calls(cuda_ok):
    import torch
    P = pkg()
    L = P.load_library()
    rng = np.random.default_rng(31)
    # two calls in a row with different sizes, then one that fills the scratch exactly
    # (1024 x 1024 = 1,048,576 values: the last bytes of the lo half are written and read)
    for rows, cols, m in ((960, 576, 9), (576, 1536, 64), (64, 1024, 1024)):
        packed, sc, x = _case(rng, rows, cols, m)
        dp, ds, dx = (torch.from_numpy(a).cuda() for a in (packed, sc, x))
        y_ref = torch.empty((m, rows), dtype=torch.float32, device="cuda")
        y_na = torch.full((m, rows), float("nan"), dtype=torch.float32, device="cuda")
        assert L.mllm_gemm_q4(dp.data_ptr(), ds.data_ptr(), dx.data_ptr(), y_ref.data_ptr(), rows, cols, m, None) == 0
        assert L.mllm_gemm_q4_noalloc(dp.data_ptr(), ds.data_ptr(), dx.data_ptr(), y_na.data_ptr(), rows, cols, m,
                                      None) == 0
        torch.cuda.synchronize()
        a, b = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(a).all()
        assert np.abs(a - b).max() <= 1e-4 * np.abs(b).max() + 1e-6


@pytest.mark.gpu
def test_noalloc_gemm_rejects_oversize(cuda_ok):
    import torch
    P = pkg()
    L = P.load_library()
    t = torch.zeros(16, dtype=torch.float32, device="cuda")
    # 1024 rows of 2048 activations = 2,097,152 values > the 1,048,576 fixed scratch
    rc = L.mllm_gemm_q4_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 64, 2048, 1024, None)
    assert rc == -3
    assert b"1,048,576" in L.mllm_last_error(None)
