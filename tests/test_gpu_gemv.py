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
    for m in (1, 2, 4, 5, 9, 16):
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


def _dense_weights(dtype, rows, cols, rng):
    """Seeded weights of each PGW storage kind: the stored words and (q8) the per-row scales."""
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)
    if dtype == "f32":
        return w, None
    if dtype == "f16":
        return w.astype(np.float16).view(np.uint16), None
    if dtype == "bf16":  # round to nearest even on the top 16 bits
        u = w.view(np.uint32).astype(np.uint64)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16), None
    amax = np.abs(w).max(axis=1)
    sc = np.where(amax > 0, amax / 127.0, 1.0).astype(np.float32)
    return np.clip(np.rint(w / sc[:, None]), -127, 127).astype(np.int8), sc


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16", "q8"])
@pytest.mark.parametrize("rows,cols", [(576, 576), (1536, 576), (576, 1536), (49152, 576)])
def test_gemv_dense_matches_oracle(dtype, rows, cols, cuda_ok):
    """mllm_gemv against gemvF32 / gemvF16 / gemvBf16 / gemvQ8 (engine/infer.js:10-86), M in {1, 5, 16}."""
    import torch
    P = pkg()
    rng = np.random.default_rng(7)
    w, sc = _dense_weights(dtype, rows, cols, rng)
    dw = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    ds = torch.from_numpy(sc).cuda() if sc is not None else None
    idx = np.arange(0, rows, max(1, rows // 512))
    for m in (1, 5, 16):
        x = rng.standard_normal((m, cols), dtype=np.float32)
        dx = torch.from_numpy(x).cuda()
        dy = torch.empty((m, rows), dtype=torch.float32, device="cuda")
        P.gemv_device(dtype, dw.data_ptr(), ds.data_ptr() if ds is not None else 0, dx.data_ptr(), dy.data_ptr(),
                      rows, cols, m)
        torch.cuda.synchronize()
        y = dy.cpu().numpy()
        for i in range(m):
            ref = O.gemv_dense(dtype, w[idx], sc[idx] if sc is not None else None, x[i])
            err = np.abs(y[i, idx] - ref).max()
            assert err <= 1e-4 * np.abs(ref).max() + 1e-6, (dtype, rows, cols, m, i, err)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16", "q8"])
def test_gemv_dense_ragged_rows(dtype, cuda_ok):
    """Row counts that leave a warp's last rows empty (13, 1) and activation counts below the kernel's
    tile (3 of 4, 7 of 8, 11 of 16), against the oracle."""
    import torch
    P = pkg()
    rng = np.random.default_rng(9)
    for rows, cols in ((13, 64), (1, 32), (37, 96)):
        w, sc = _dense_weights(dtype, rows, cols, rng)
        dw = torch.from_numpy(np.ascontiguousarray(w)).cuda()
        ds = torch.from_numpy(sc).cuda() if sc is not None else None
        for m in (3, 7, 11):
            x = rng.standard_normal((m, cols), dtype=np.float32)
            dx = torch.from_numpy(x).cuda()
            dy = torch.full((m, rows), float("nan"), dtype=torch.float32, device="cuda")
            P.gemv_device(dtype, dw.data_ptr(), ds.data_ptr() if ds is not None else 0, dx.data_ptr(),
                          dy.data_ptr(), rows, cols, m)
            torch.cuda.synchronize()
            y = dy.cpu().numpy()
            for i in range(m):
                ref = O.gemv_dense(dtype, w, sc, x[i])
                err = np.abs(y[i] - ref).max()
                assert err <= 1e-4 * np.abs(ref).max() + 1e-6, (dtype, rows, cols, m, i, err)


@pytest.mark.gpu
def test_gemv_dense_rejects_bad_arguments(cuda_ok):
    import torch
    P = pkg()
    L = P.load_library()
    t = torch.zeros(4096, dtype=torch.float32, device="cuda")
    p = t.data_ptr()
    assert L.mllm_gemv(4, p, p, p, p, 4, 64, 1, None) == -2   # q4: mllm_gemv_q4's layout
    assert L.mllm_gemv(7, p, p, p, p, 4, 64, 1, None) == -3   # no such storage kind
    assert L.mllm_gemv(1, p, p, p, p, 4, 12, 1, None) == -3   # f16 rows of 24 bytes: not whole chunks
    assert L.mllm_gemv(0, p, p, p, p, 4, 64, 17, None) == -3  # n_act > 16
    assert L.mllm_gemv(3, p, None, p, p, 4, 64, 1, None) == -3  # q8 without its row scales
    assert L.mllm_gemv(0, p + 4, p, p, p, 4, 64, 1, None) == -3  # misaligned weights
