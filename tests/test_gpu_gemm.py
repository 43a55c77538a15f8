"""Tensor-core Q4 GEMM (mllm_gemm_q4) against the f64 product of the dequantised weights
(engine/infer.js:88-116 per activation row; the oracle's gemvQ4 on a row sample for the small case).

Tolerance: |y - y_ref| <= 1e-4 * max|y_ref| + 1e-6 (fp32 accumulation, fp16 hi+lo activations)."""
import numpy as np
import pytest

from conftest import pkg
from oracle import oracle as O

SHAPES = [(576, 576), (192, 576), (1536, 576), (576, 1536), (960, 960), (2560, 960), (960, 2560), (49152, 576),
          (100, 64)]


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_gemm_q4_matches_reference(rows, cols, cuda_ok):
    import torch
    P = pkg()
    rng = np.random.default_rng(2)
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    packed, sc = P.quant_q4(w)
    wd = P.dequant_q4(packed, sc).astype(np.float64)
    dp, ds = torch.from_numpy(packed).cuda(), torch.from_numpy(sc).cuda()
    # up to 16 rows: the mma.sync tile; 24, 40, 67, 256: tcgen05 token tiles of 32, 64 and 128; 1,024 rows
    # of the (2560, 960) shape: 256-token tiles (the 128-token grid would exceed one wave of 148 CTAs)
    ms = (1, 5, 9, 16, 24, 40, 67, 256) + ((1024,) if (rows, cols) == (2560, 960) else ())
    for m in ms:
        if rows * m > 49152 * 16 and m > 16:
            continue
        x = rng.standard_normal((m, cols), dtype=np.float32)
        x[:, :7] *= np.float32(1e-3)  # small activations exercise the fp16 lo half
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty((m, rows), dtype=torch.float32, device="cuda")
        P.gemm_q4_device(dp.data_ptr(), ds.data_ptr(), dx.data_ptr(), dy.data_ptr(), rows, cols, m)
        torch.cuda.synchronize()
        y = dy.cpu().numpy()
        ref = x.astype(np.float64) @ wd.T
        err = np.abs(y - ref).max()
        assert err <= 1e-4 * np.abs(ref).max() + 1e-6, (rows, cols, m, err)
    # oracle spot check on one row of activations
    idx = np.arange(0, rows, max(1, rows // 64))
    np.testing.assert_allclose(y[0, idx], O.gemv_q4(packed[idx], sc[idx], x[0]), rtol=0, atol=1e-4 * np.abs(ref).max())
