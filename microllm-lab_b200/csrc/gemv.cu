// Standalone Q4 group-32 GEMV / skinny GEMM (M <= 16 activation rows) on CUDA cores:
// y[m][r] = sum_g sc[r][g] * sum_k (q[r][32g+k] - 8) * x[m][32g+k]   (engine/infer.js:88-116).
//
// Streaming design: each warp owns ROWS consecutive rows; every lane issues all of its 4-byte weight
// loads (and scale loads) for those rows before the first FMA, so a CTA keeps
// 8 warps x ROWS x cols/2 bytes in flight.  Activations are read through the read-only cache (they
// are small and shared by every row).  fp32 accumulation.
#include <cuda_runtime.h>

#include <algorithm>

#include "../../include/mllm.h"
#include "device_common.cuh"

namespace mllm {

template <int NWJ, int ROWS, int MT>
__global__ void __launch_bounds__(256) gemv_q4_kernel(const uint32_t* __restrict__ W, const float* __restrict__ S,
                                                      const float* __restrict__ X, float* __restrict__ Y, int R, int n,
                                                      int M) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int nwords = n >> 3;
  for (int r0 = warp * ROWS; r0 < R; r0 += nwarps * ROWS) {
    uint32_t w[ROWS][NWJ];
    float s[ROWS][NWJ];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
      const int r = r0 + i;
#pragma unroll
      for (int j = 0; j < NWJ; ++j) {
        const int k = lane + 32 * j;
        const bool ok = r < R && k < nwords;
        w[i][j] = ok ? __ldcs(W + (size_t)r * nwords + k) : 0x88888888u;
        s[i][j] = ok ? __ldcs(S + (size_t)r * (nwords >> 2) + (k >> 2)) : 0.f;
      }
    }
    float acc[ROWS][MT];
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[i][m] = 0.f;
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      if (k >= nwords) break;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= M) break;
        const float4 xa = __ldg(reinterpret_cast<const float4*>(X + (size_t)m * n + 8 * k));
        const float4 xb = __ldg(reinterpret_cast<const float4*>(X + (size_t)m * n + 8 * k + 4));
#pragma unroll
        for (int i = 0; i < ROWS; ++i) {
          const uint32_t lo = w[i][j] & 0x0F0F0F0Fu, hi = (w[i][j] >> 4) & 0x0F0F0F0Fu;
          float t = nib_at(lo, 0) * xa.x;
          t = fmaf(nib_at(hi, 0), xa.y, t);
          t = fmaf(nib_at(lo, 1), xa.z, t);
          t = fmaf(nib_at(hi, 1), xa.w, t);
          t = fmaf(nib_at(lo, 2), xb.x, t);
          t = fmaf(nib_at(hi, 2), xb.y, t);
          t = fmaf(nib_at(lo, 3), xb.z, t);
          t = fmaf(nib_at(hi, 3), xb.w, t);
          acc[i][m] = fmaf(t, s[i][j], acc[i][m]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < ROWS; ++i) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m >= M) break;
        const float v = warp_sum(acc[i][m]);
        if (lane == 0 && r0 + i < R) Y[(size_t)m * R + r0 + i] = v;
      }
    }
  }
}

template <int NWJ, int ROWS, int MT>
static cudaError_t run_gemv(const uint32_t* W, const float* S, const float* X, float* Y, int R, int n, int M,
                            cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int warps_needed = (R + ROWS - 1) / ROWS;
  const int blocks = std::max(1, std::min((warps_needed + 7) / 8, sms * 8));
  gemv_q4_kernel<NWJ, ROWS, MT><<<blocks, 256, 0, st>>>(W, S, X, Y, R, n, M);
  return cudaGetLastError();
}

template <int NWJ>
static cudaError_t dispatch_m(const uint32_t* W, const float* S, const float* X, float* Y, int R, int n, int M,
                              cudaStream_t st) {
  if (M == 1) return run_gemv<NWJ, 4, 1>(W, S, X, Y, R, n, M, st);
  if (M <= 4) return run_gemv<NWJ, 2, 4>(W, S, X, Y, R, n, M, st);
  if (M <= 8) return run_gemv<NWJ, 2, 8>(W, S, X, Y, R, n, M, st);
  return run_gemv<NWJ, 1, 16>(W, S, X, Y, R, n, M, st);
}

}  // namespace mllm

extern "C" int mllm_gemv_q4(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y, int rows,
                            int cols, int n_act, void* stream) {
  using namespace mllm;
  if (!d_packed || !d_scales || !d_x || !d_y || rows <= 0 || cols <= 0 || cols % 32 || n_act < 1 || n_act > 16)
    return MLLM_ERR_ARG;
  if (((uintptr_t)d_packed & 3) || ((uintptr_t)d_x & 15)) return MLLM_ERR_ARG;
  const uint32_t* W = reinterpret_cast<const uint32_t*>(d_packed);
  cudaStream_t st = (cudaStream_t)stream;
  const int nwj = (cols / 8 + 31) / 32;
  cudaError_t e;
  if (nwj <= 1) e = dispatch_m<1>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else if (nwj <= 2) e = dispatch_m<2>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else if (nwj <= 3) e = dispatch_m<3>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else if (nwj <= 4) e = dispatch_m<4>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else if (nwj <= 8) e = dispatch_m<8>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else if (nwj <= 12) e = dispatch_m<12>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else if (nwj <= 16) e = dispatch_m<16>(W, d_scales, d_x, d_y, rows, cols, n_act, st);
  else return MLLM_ERR_UNSUPPORTED;
  return e == cudaSuccess ? MLLM_OK : MLLM_ERR_CUDA;
}
