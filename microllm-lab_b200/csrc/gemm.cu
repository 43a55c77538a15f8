// Q4 GEMM over T activation rows on the tensor cores (mllm_gemm_q4): the batched / skinny form of
// gemvQ4 (engine/infer.js:88-116) used for prefill, verify and multi-sequence decode.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/mllm.h"
#include "q4mma.cuh"

namespace mllm {

// f32 [T][K] -> fp16 hi, lo [T][K]
__global__ void split_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    __half h, l;
    split_hi_lo(x[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

template <int TBW>
__global__ void __launch_bounds__(kGemmThreads) gemm_store_kernel(const uint8_t* W, const float* S, const __half* xh,
                                                                  const __half* xl, float* Y, int R, int K, int T) {
  extern __shared__ __align__(16) unsigned char smem[];
  q4_gemm_tile<TBW>(W, S, xh, xl, K, R, K, T, blockIdx.x * kGemmRows, blockIdx.y * 8 * TBW, smem,
                    [&](int r, int t, float v) { Y[(size_t)t * R + r] = v; });
}

cudaError_t launch_gemm_store(const uint8_t* W, const float* S, const __half* xh, const __half* xl, float* Y, int R,
                              int K, int T, cudaStream_t st) {
  const dim3 grid((R + kGemmRows - 1) / kGemmRows, 1);
  if (T <= 16) {
    constexpr size_t sm = q4_gemm_smem_bytes<2>();
    gemm_store_kernel<2><<<dim3(grid.x, (T + 15) / 16), kGemmThreads, sm, st>>>(W, S, xh, xl, Y, R, K, T);
  } else {
    constexpr size_t sm = q4_gemm_smem_bytes<8>();
    gemm_store_kernel<8><<<dim3(grid.x, (T + 63) / 64), kGemmThreads, sm, st>>>(W, S, xh, xl, Y, R, K, T);
  }
  return cudaGetLastError();
}

cudaError_t launch_split(const float* x, __half* hi, __half* lo, size_t n, cudaStream_t st) {
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  split_kernel<<<blocks, 256, 0, st>>>(x, hi, lo, n);
  return cudaGetLastError();
}

namespace {
// Per-device workspace for the fp16 halves of the activations (grown on demand, kept until exit).
struct Workspace {
  std::mutex mu;
  std::vector<void*> ptr;
  std::vector<size_t> cap;
};
Workspace g_ws;

int workspace(size_t bytes, __half** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MLLM_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_ws.mu);
  if ((int)g_ws.ptr.size() <= dev) {
    g_ws.ptr.resize(dev + 1, nullptr);
    g_ws.cap.resize(dev + 1, 0);
  }
  if (g_ws.cap[dev] < bytes) {
    if (g_ws.ptr[dev]) {
      cudaDeviceSynchronize();
      cudaFree(g_ws.ptr[dev]);
    }
    g_ws.ptr[dev] = nullptr;
    g_ws.cap[dev] = 0;
    if (cudaMalloc(&g_ws.ptr[dev], bytes) != cudaSuccess) return MLLM_ERR_OOM;
    g_ws.cap[dev] = bytes;
  }
  *out = (__half*)g_ws.ptr[dev];
  return MLLM_OK;
}
}  // namespace

}  // namespace mllm

extern "C" int mllm_gemm_q4(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y, int rows,
                            int cols, int n_act, void* stream) {
  using namespace mllm;
  if (!d_packed || !d_scales || !d_x || !d_y || rows <= 0 || cols <= 0 || cols % 32 || n_act <= 0) return MLLM_ERR_ARG;
  if (((uintptr_t)d_packed & 15) || ((uintptr_t)d_scales & 3) || ((uintptr_t)d_x & 3)) return MLLM_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t n = (size_t)n_act * cols;
  __half* ws = nullptr;
  int rc = workspace(2 * n * sizeof(__half) + 256, &ws);
  if (rc) return rc;
  __half* hi = ws;
  __half* lo = ws + ((n + 127) / 128) * 128;
  if (launch_split(d_x, hi, lo, n, st) != cudaSuccess) return MLLM_ERR_CUDA;
  if (launch_gemm_store(d_packed, d_scales, hi, lo, d_y, rows, cols, n_act, st) != cudaSuccess) return MLLM_ERR_CUDA;
  return MLLM_OK;
}
