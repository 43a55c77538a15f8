// Matrix-vector / skinny-matrix products for the PGW storage kinds other than q4: the row loops
// gemvF32, gemvF16, gemvBf16 and gemvQ8 of engine/infer.js:10-86, which the engine binds per tensor
// storage in _bindGemv / gemv (engine/infer.js:314-345).
//
// y[a][r] = sum_k W[r][k] x[a][k] for a < n_act (q8: times the row scale after the sum, as gemvQ8 does),
// fp32 accumulation.  One warp per four weight rows (two above 8 activation rows): lane l streams
// 16-byte chunks l, l + 32, ... of the rows (4 f32, 8 f16 / bf16 or 16 int8 weights each), converts
// them exactly to f32 and multiplies them into every activation row, each activation load (through L1:
// all warps read the same rows) serving all the warp's rows; the 32 lane sums of each (row, activation
// row) meet in a fixed xor-shuffle tree.  The weight bytes are read once, so the kernel is bound by HBM
// (or L2) bandwidth for large matrices and by launch latency for small ones.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/mllm.h"
#include "device_common.cuh"

namespace mllm {
namespace {

constexpr int kDenseWarps = 8;

// Bytes per weight of each storage kind (MLLM_DTYPE_*).
__host__ __device__ constexpr int dense_esize(int dt) { return dt == MLLM_DTYPE_F32 ? 4 : (dt == MLLM_DTYPE_Q8 ? 1 : 2); }

// Weights 4 q .. 4 q + 3 of the 16-byte chunk v as f32 (exact for every kind).
template <int DT>
__device__ __forceinline__ float4 dense_w4(const uint4 v, int q) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
  if constexpr (DT == MLLM_DTYPE_F32) {
    return make_float4(__uint_as_float(u[0]), __uint_as_float(u[1]), __uint_as_float(u[2]), __uint_as_float(u[3]));
  } else if constexpr (DT == MLLM_DTYPE_F16) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u[2 * q]));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u[2 * q + 1]));
    return make_float4(a.x, a.y, b.x, b.y);
  } else if constexpr (DT == MLLM_DTYPE_BF16) {  // engine/infer.js:66-77: the 16 bits are the top of an f32
    const uint32_t a = u[2 * q], b = u[2 * q + 1];
    return make_float4(__uint_as_float(a << 16), __uint_as_float(a & 0xFFFF0000u), __uint_as_float(b << 16),
                       __uint_as_float(b & 0xFFFF0000u));
  } else {  // q8: signed bytes
    const uint32_t a = u[q];
    return make_float4((float)(int8_t)a, (float)(int8_t)(a >> 8), (float)(int8_t)(a >> 16), (float)(int8_t)(a >> 24));
  }
}

// The weight rows per warp share every activation load; lane l streams 16-byte chunks l, l + 32, ... of
// those rows.
__host__ __device__ constexpr int dense_rows(int m) { return m > 8 ? 2 : 4; }
template <int DT, int M>
__global__ void __launch_bounds__(kDenseWarps * 32) gemv_dense_kernel(const uint8_t* __restrict__ W,
                                                                      const float* __restrict__ S,
                                                                      const float* __restrict__ x,
                                                                      float* __restrict__ y, int rows, int cols,
                                                                      int n_act) {
  constexpr int E = 16 / dense_esize(DT);  // weights per chunk
  constexpr int RW = dense_rows(M);
  const int lane = threadIdx.x & 31;
  const int r0 = (blockIdx.x * kDenseWarps + (threadIdx.x >> 5)) * RW;
  if (r0 >= rows) return;
  const int nch = cols / E;  // chunks per row
  const size_t rbytes = (size_t)cols * dense_esize(DT);
  const uint4* wr[RW];
#pragma unroll
  for (int j = 0; j < RW; ++j)  // rows past the matrix re-read the last row (their sums are dropped)
    wr[j] = reinterpret_cast<const uint4*>(W + (size_t)min(r0 + j, rows - 1) * rbytes);
  float acc[RW][M];
#pragma unroll
  for (int j = 0; j < RW; ++j)
#pragma unroll
    for (int a = 0; a < M; ++a) acc[j][a] = 0.f;
  for (int c = lane; c < nch; c += 32) {
    uint4 v[RW];
#pragma unroll
    for (int j = 0; j < RW; ++j) v[j] = __ldg(wr[j] + c);
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      float4 w4[RW];
#pragma unroll
      for (int j = 0; j < RW; ++j) w4[j] = dense_w4<DT>(v[j], q);
#pragma unroll
      for (int a = 0; a < M; ++a) {
        if (a >= n_act) break;
        const float4 xv = __ldg(reinterpret_cast<const float4*>(x + (size_t)a * cols + (size_t)c * E) + q);
#pragma unroll
        for (int j = 0; j < RW; ++j) {
          acc[j][a] = fmaf(w4[j].x, xv.x, acc[j][a]);
          acc[j][a] = fmaf(w4[j].y, xv.y, acc[j][a]);
          acc[j][a] = fmaf(w4[j].z, xv.z, acc[j][a]);
          acc[j][a] = fmaf(w4[j].w, xv.w, acc[j][a]);
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < RW; ++j) {
    const int r = r0 + j;
    const float sc = DT == MLLM_DTYPE_Q8 && r < rows ? __ldg(S + r) : 1.f;
#pragma unroll
    for (int a = 0; a < M; ++a) {
      if (a >= n_act) break;
      const float s = warp_sum(acc[j][a]);
      if (lane == 0 && r < rows) y[(size_t)a * rows + r] = DT == MLLM_DTYPE_Q8 ? s * sc : s;
    }
  }
}

template <int DT>
cudaError_t launch_dense(const uint8_t* W, const float* S, const float* x, float* y, int rows, int cols, int n_act,
                         cudaStream_t st) {
  const int M = n_act <= 1 ? 1 : (n_act <= 4 ? 4 : (n_act <= 8 ? 8 : 16));
  const int per_cta = kDenseWarps * dense_rows(M);
  const dim3 grid((rows + per_cta - 1) / per_cta), block(kDenseWarps * 32);
  if (M == 1)
    gemv_dense_kernel<DT, 1><<<grid, block, 0, st>>>(W, S, x, y, rows, cols, n_act);
  else if (M == 4)
    gemv_dense_kernel<DT, 4><<<grid, block, 0, st>>>(W, S, x, y, rows, cols, n_act);
  else if (M == 8)
    gemv_dense_kernel<DT, 8><<<grid, block, 0, st>>>(W, S, x, y, rows, cols, n_act);
  else
    gemv_dense_kernel<DT, 16><<<grid, block, 0, st>>>(W, S, x, y, rows, cols, n_act);
  return cudaGetLastError();
}

}  // namespace
}  // namespace mllm

extern "C" int mllm_gemv(int dtype, const void* d_w, const float* d_scales, const float* d_x, float* d_y, int rows,
                         int cols, int n_act, void* stream) {
  using namespace mllm;
  if (dtype == MLLM_DTYPE_Q4) return MLLM_ERR_UNSUPPORTED;  // mllm_gemv_q4 takes the packed layout
  if (dtype < MLLM_DTYPE_F32 || dtype > MLLM_DTYPE_Q8) return MLLM_ERR_ARG;
  if (!d_w || !d_x || !d_y || rows <= 0 || cols <= 0 || n_act < 1 || n_act > 16) return MLLM_ERR_ARG;
  if (dtype == MLLM_DTYPE_Q8 && !d_scales) return MLLM_ERR_ARG;
  // whole 16-byte chunks per row, 16-byte aligned rows and activations
  if ((cols * dense_esize(dtype)) % 16 || cols % 4 || ((uintptr_t)d_w & 15) || ((uintptr_t)d_x & 15)) return MLLM_ERR_ARG;
  const uint8_t* W = static_cast<const uint8_t*>(d_w);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  switch (dtype) {
    case MLLM_DTYPE_F32: e = launch_dense<MLLM_DTYPE_F32>(W, d_scales, d_x, d_y, rows, cols, n_act, st); break;
    case MLLM_DTYPE_F16: e = launch_dense<MLLM_DTYPE_F16>(W, d_scales, d_x, d_y, rows, cols, n_act, st); break;
    case MLLM_DTYPE_BF16: e = launch_dense<MLLM_DTYPE_BF16>(W, d_scales, d_x, d_y, rows, cols, n_act, st); break;
    default: e = launch_dense<MLLM_DTYPE_Q8>(W, d_scales, d_x, d_y, rows, cols, n_act, st); break;
  }
  return e == cudaSuccess ? MLLM_OK : MLLM_ERR_CUDA;
}
