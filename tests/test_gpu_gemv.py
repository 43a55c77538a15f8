"""Q4 GEMV / skinny-matrix kernel (mllm_gemv_q4) against the oracle's gemvQ4 (engine/infer.js:88-116).

Tolerance: fp32 accumulation against the f64 oracle, |y - y_ref| <= 1e-4 * max|y_ref| + 1e-6."""
import numpy as np
import pytest

from conftest import pkg
from oracle import oracle as O

SHAPES = [(576, 576), (192, 576), (1536, 576), (576, 1536), (960, 960), (2560, 960), (960, 2560), (49152, 576)]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemv_q4_matches_oracle(rows, cols, cuda_ok):
    import torch
    P = pkg()
    rng = np.random.default_rng(1)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    packed, sc = P.quant_q4(w)
    dp = torch.from_numpy(packed).cuda()
    ds = torch.from_numpy(sc).cuda()
    for m in (1, 5, 9, 16):
        x = rng.standard_normal((m, cols), dtype=np.float32)
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty((m, rows), dtype=torch.float32, device="cuda")
        P.gemv_q4_device(dp.data_ptr(), ds.data_ptr(), dx.data_ptr(), dy.data_ptr(), rows, cols, m)
        torch.cuda.synchronize()
        y = dy.cpu().numpy()
        idx = np.arange(0, rows, max(1, rows // 512))  # oracle on a row sample for the big shape
        for i in range(m):
            ref = O.gemv_q4(packed[idx], sc[idx], x[i])
            err = np.abs(y[i, idx] - ref).max()
            assert err <= 1e-4 * np.abs(ref).max() + 1e-6, (rows, cols, m, i, err)


@pytest.mark.gpu
def test_gemv_q4_rejects_bad_arguments(cuda_ok):
    import torch
    P = pkg()
    L = P.load_library()
    t = torch.zeros(64, dtype=torch.float32, device="cuda")
    assert L.mllm_gemv_q4(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 4, 48, 1, None) == -3  # cols % 32
    assert L.mllm_gemv_q4(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), 4, 32, 17, None) == -3  # n_act > 16
