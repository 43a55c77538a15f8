// Q4 GEMM on the 5th-generation tensor cores for mllm_gemm_q4: Y[T][R] = X[T][K] . W^T (the tile and its
// precision scheme are in tc5.cuh).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "tc5.cuh"

namespace mllm {

using namespace tc5;

__device__ int g_tc5_error;  // set when a wait of gemm_tc5_kernel ran out its limit

// grid (ceil(R / 128), ceil(T / N)), kTc5Threads + 64 threads; dynamic shared memory
// tc5_smem_bytes<N, S>().  xh / xl are the activation halves in the tiled layout of split_tiled_kernel.
template <int N, int S>
__global__ void __launch_bounds__(kTc5Threads + 64, 1) gemm_tc5_kernel(const uint8_t* __restrict__ W,
                                                                      const float* __restrict__ Sc,
                                                                      const __half* __restrict__ xh,
                                                                      const __half* __restrict__ xl,
                                                                      float* __restrict__ Y, int R, int K, int T,
                                                                      int T8) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int r0 = blockIdx.x * kTc5Rows, t0 = blockIdx.y * N;
  const Tc5Acc acc = tc5_tile<N, S>(W, Sc, xh, xl, R, K, T8, r0, t0, smem, false, &g_tc5_error);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (acc.ok && warp < kTc5Threads / 32) {
    // warp w: rows 32 (w % 4) + lane, column half w / 4
    constexpr int kHalf = N >= 32 ? N / 2 : N;
    const int cbeg = (warp >> 2) * kHalf;
    const int erow = r0 + (warp & 3) * 32 + lane;
#pragma unroll
    for (int c0 = cbeg; c0 < cbeg + kHalf && c0 < N; c0 += 16) {
      float v[16];
      tc5_cols16<N>(acc, warp, c0, v);
      if (erow < R)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = t0 + c0 + i;
          if (t < T) Y[(size_t)t * R + erow] = v[i];
        }
    }
  }
  tc5_release<N>(acc);
}

// f32 [T][K] -> the tiled fp16 hi / lo halves gemm_tc5_kernel reads (tiled_at): thread i converts token
// 8 t8 + n8, columns 32 g + 8 c .. + 7 with i = ((g T8 + t8) 4 + c) 8 + n8.  Tokens past T are 0.
__global__ void split_tiled_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo,
                                   int T, int K, int T8, bool vec) {
  const size_t n = (size_t)T8 * 8 * (K / 8);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int n8 = (int)(i & 7), c = (int)((i >> 3) & 3);
    const size_t rest = i >> 5;
    const int t8 = (int)(rest % T8), g = (int)(rest / T8);
    const int t = 8 * t8 + n8;
    float v[8];
    if (t < T) {
      const float* p = x + (size_t)t * K + 32 * g + 8 * c;
      if (vec) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p + 4));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldg(p + j);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = 0.f;
    }
    __half2 h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
      const float2 hf = __half22float2(h[j]);
      l[j] = __floats2half2_rn(v[2 * j] - hf.x, v[2 * j + 1] - hf.y);
    }
    const size_t o = tiled_at(t, 32 * g + 8 * c, T8);  // the chunk's place in its swizzled block
    *reinterpret_cast<uint4*>(hi + o) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(lo + o) = *reinterpret_cast<const uint4*>(l);
  }
}

template <int N, int S>
static cudaError_t launch_tc5(const uint8_t* W, const float* Sc, const __half* xh, const __half* xl, float* Y, int R,
                              int K, int T, cudaStream_t st) {
  constexpr size_t sm = tc5_smem_bytes<N, S>();
  static bool init = false;  // the attribute is per function; set once per process
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc5_kernel<N, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    init = true;
  }
  const dim3 grid((R + kTc5Rows - 1) / kTc5Rows, (T + N - 1) / N);
  gemm_tc5_kernel<N, S><<<grid, kTc5Threads + 64, sm, st>>>(W, Sc, xh, xl, Y, R, K, T, (T + 7) / 8);
  return cudaGetLastError();
}

// Halves (in elements) of one tiled activation array for T tokens of K columns.
size_t tc5_tiled_halves(int T, int K) { return (size_t)((T + 7) / 8) * 8 * K; }

cudaError_t launch_split_tiled(const float* x, __half* hi, __half* lo, int T, int K, cudaStream_t st) {
  const size_t n = tc5_tiled_halves(T, K) / 8;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  split_tiled_kernel<<<blocks, 256, 0, st>>>(x, hi, lo, T, K, (T + 7) / 8, ((uintptr_t)x & 15) == 0);
  return cudaGetLastError();
}

// Y[T][R] for K a multiple of 32 from the tiled halves.  A CTA's time is set by its K loop (about
// 600 cycles per group, the dequantisation), nearly independent of N up to 128, so the tiles are as
// wide as possible: N = 128 for more than 64 tokens, N = 256 once the 128-token grid would take more
// than one wave of 148 CTAs (the tensor pipe then sets the pace, and half as many CTAs run).  Up to 64
// tokens one tile of 16, 32 or 64 covers them, two CTAs per SM.
cudaError_t launch_gemm_tc5(const uint8_t* W, const float* Sc, const __half* xh, const __half* xl, float* Y, int R,
                            int K, int T, cudaStream_t st) {
  const long rt = (R + kTc5Rows - 1) / kTc5Rows;
  if (T > 128 && rt * ((T + 127) / 128) > 148) return launch_tc5<256, 4>(W, Sc, xh, xl, Y, R, K, T, st);
  if (T > 64) return launch_tc5<128, 6>(W, Sc, xh, xl, Y, R, K, T, st);
  if (T > 32) return launch_tc5<64, 4>(W, Sc, xh, xl, Y, R, K, T, st);
  if (T > 16) return launch_tc5<32, 5>(W, Sc, xh, xl, Y, R, K, T, st);
  return launch_tc5<16, 6>(W, Sc, xh, xl, Y, R, K, T, st);
}

}  // namespace mllm
