// Q4 GEMM on the 5th-generation tensor cores (tcgen05.mma, accumulator in tensor memory) for
// mllm_gemm_q4: Y[T][R] = X[T][K] . W^T with W the PGW Q4 rows (engine/infer.js:88-116 per activation
// row).
//
// One CTA (128 threads) computes a 128-row x N-token tile.  The K loop walks the Q4 groups (32 columns):
// every thread dequantises one weight row's group into shared memory, the 32 x N activation halves come
// in by cp.async, and thread 0 issues the group's MMAs; a ring of kTc5Stages stages lets the next
// groups' dequantisation overlap the MMAs in flight (tcgen05.commit releases a stage on its mbarrier).
//
// Precision.  The group scale is folded into the weights, w = (q - 8) s 2^E (2^E per CTA puts the
// tile's largest |w| near 2^14, so that the fp16 low halves stay normal), and both operands are split
// into fp16 hi + lo halves (x = hi + lo with |lo| <= 2^-11 |x|).  The accumulator takes
// w_hi x_hi + w_hi x_lo + w_lo x_hi in fp32; the dropped w_lo x_lo term is below 2^-22 of each product.
// The epilogue scales by 2^-E (exact).
//
// Operand layout in shared memory (K-major, no swizzle, the UMMA canonical interleaved form): an 8-row x
// 16-byte core matrix is 128 contiguous bytes; core matrices along K are kTc5Lbo bytes apart, along
// M / N kTc5Sbo bytes apart, so element (row, k) of a 32-column stage sits at
// (row / 8) kTc5Sbo + (k / 8) kTc5Lbo + (row % 8) 16 + (k % 8) 2.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "device_common.cuh"

namespace mllm {
namespace tc5 {

constexpr int kTc5Rows = 128;    // M: weight rows per CTA
constexpr int kTc5Threads = 128;
constexpr int kTc5Stages = 4;
constexpr int kTc5Lbo = 128;     // bytes between core matrices along K
constexpr int kTc5Sbo = 512;     // bytes between core matrices along M / N (4 along K per stage)
constexpr int kTc5ABytes = kTc5Rows * 32 * 2;  // one fp16 half of a stage's weights: 8 KB

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor (K-major, no swizzle, version 1).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((kTc5Lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((kTc5Sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 accumulator, M = 128, N.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTc5Rows >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t dtmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(dtmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_wait_upto(int n) {
  switch (n) {
    case 0: cp_wait<0>(); break;
    case 1: cp_wait<1>(); break;
    case 2: cp_wait<2>(); break;
    default: cp_wait<3>(); break;
  }
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, uint64_t limit) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (globaltimer() - t0 > limit) return false;
  }
}

}  // namespace tc5

using namespace tc5;

__device__ int g_tc5_error;  // set when a wait of gemm_tc5_kernel ran out its limit

// grid (ceil(R / 128), ceil(T / N)); dynamic shared memory: kTc5Stages x (2 x 8 KB + 2 x N x 64 B).
template <int N>
__global__ void __launch_bounds__(kTc5Threads, 1) gemm_tc5_kernel(const uint8_t* __restrict__ W,
                                                                 const float* __restrict__ S,
                                                                 const __half* __restrict__ xh,
                                                                 const __half* __restrict__ xl, float* __restrict__ Y,
                                                                 int R, int K, int T) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kB = N * 32 * 2;                    // one fp16 half of a stage's activations
  constexpr int kStage = 2 * kTc5ABytes + 2 * kB;
  __shared__ __align__(8) uint64_t bars[kTc5Stages];
  __shared__ uint32_t tmem_base;
  __shared__ float smax[kTc5Threads / 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = blockIdx.x * kTc5Rows, t0 = blockIdx.y * N, NG = K / 32;
  const int row = r0 + tid;
  const bool row_ok = row < R;
  const uint64_t limit = kWaitNs;
  constexpr uint32_t kCols = N < 32 ? 32 : N;  // tensor-memory columns (a power of 2 >= 32)

  // ---- tensor memory for the accumulator (warp 0), barriers, the tile's power-of-two weight scale
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < kTc5Stages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&bars[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  float m = 0.f;
  if (row_ok)
    for (int g = 0; g < NG; ++g) m = fmaxf(m, fabsf(S[(size_t)row * NG + g]));
  m = warp_max(m);
  if (lane == 0) smax[warp] = m;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t dtmem = tmem_base;
  m = fmaxf(fmaxf(smax[0], smax[1]), fmaxf(smax[2], smax[3]));
  int e2 = 0;
  if (m > 0.f) (void)frexpf(8.f * m, &e2);  // 8 m < 2^e2
  const int E = 14 - e2;                      // |w| 2^E < 2^14
  const float up = ldexpf(1.f, E), down = ldexpf(1.f, -E);
  const uint32_t idesc = idesc_f16(N);
  const uint8_t* wrow = W + (size_t)row * (K / 2);
  const float* srow = S + (size_t)row * NG;
  bool ok = true;

  // stage s: A_hi, A_lo (8 KB each), B_hi, B_lo (kB each)
  auto produce = [&](int g, int s) {
    uint8_t* st = smem + (size_t)s * kStage;
    // weights: this thread's row, group g -> 32 hi + 32 lo halves (rows past R are zero)
    uint4 q = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
    float sc = 0.f;
    if (row_ok) {
      q = *reinterpret_cast<const uint4*>(wrow + 16 * g);
      sc = srow[g] * up;
    }
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    const int rb = (tid >> 3) * kTc5Sbo + (tid & 7) * 16;
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // 8 columns: byte b of word c holds columns 8c + 2b (low) and 8c + 2b + 1
      __half2 hi[4], lo[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t byte = (qw[c] >> (8 * b)) & 0xFFu;
        const float v0 = (float)((int)(byte & 15u) - 8) * sc, v1 = (float)((int)(byte >> 4) - 8) * sc;
        const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
        hi[b] = __halves2half2(h0, h1);
        lo[b] = __halves2half2(__float2half_rn(v0 - __half2float(h0)), __float2half_rn(v1 - __half2float(h1)));
      }
      *reinterpret_cast<uint4*>(st + rb + c * kTc5Lbo) = *reinterpret_cast<const uint4*>(hi);
      *reinterpret_cast<uint4*>(st + kTc5ABytes + rb + c * kTc5Lbo) = *reinterpret_cast<const uint4*>(lo);
    }
    // activations: N token rows x 4 chunks of 8 columns, hi and lo (tokens past T are zero-filled)
    const uint32_t bh = su32(st + 2 * kTc5ABytes), bl = bh + kB;
    for (int i = tid; i < N * 4; i += kTc5Threads) {
      const int n = i >> 2, c = i & 3, t = t0 + n;
      const bool v = t < T;
      const size_t src = (size_t)(v ? t : 0) * K + 32 * g + 8 * c;
      const uint32_t off = (n >> 3) * kTc5Sbo + c * kTc5Lbo + (n & 7) * 16;
      cp16(bh + off, xh + src, v);
      cp16(bl + off, xl + src, v);
    }
    cp_commit();
  };

  for (int g = 0; g < NG + kTc5Stages - 1 && ok; ++g) {
    if (g < NG) {
      const int s = g % kTc5Stages;
      if (g >= kTc5Stages) {  // the stage's previous MMAs are done (the decision is the same in every thread)
        const bool w = bar_wait(su32(&bars[s]), ((g / kTc5Stages) - 1) & 1, limit);
        if (!__syncthreads_and(w)) {
          if (tid == 0) atomicExch(&g_tc5_error, 1);
          ok = false;
          break;
        }
      }
      produce(g, s);
    }
    const int c = g - (kTc5Stages - 1);
    if (c < 0) continue;
    cp_wait_upto(min(kTc5Stages - 1, NG - 1 - c));  // group c's copies have landed
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (tid == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t st = su32(smem + (size_t)(c % kTc5Stages) * kStage);
#pragma unroll
      for (int j = 0; j < 2; ++j) {  // two K = 16 steps of the group
        const uint64_t ah = sdesc(st + j * 2 * kTc5Lbo), al = sdesc(st + kTc5ABytes + j * 2 * kTc5Lbo);
        const uint64_t bh = sdesc(st + 2 * kTc5ABytes + j * 2 * kTc5Lbo);
        const uint64_t bl = sdesc(st + 2 * kTc5ABytes + kB + j * 2 * kTc5Lbo);
        mma_f16(dtmem, ah, bh, idesc, (c > 0 || j > 0) ? 1u : 0u);
        mma_f16(dtmem, ah, bl, idesc, 1u);
        mma_f16(dtmem, al, bh, idesc, 1u);
      }
      mma_commit(su32(&bars[c % kTc5Stages]));
    }
  }
  // ---- the last group's MMAs (and with them every earlier one) have finished: epilogue
  if (ok && !bar_wait(su32(&bars[(NG - 1) % kTc5Stages]), ((NG - 1) / kTc5Stages) & 1, limit)) {
    atomicExch(&g_tc5_error, 1);
    ok = false;
  }
  ok = __syncthreads_and(ok);
  asm volatile("cp.async.wait_all;" ::: "memory");  // no copy of this CTA is left in flight
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok) {
#pragma unroll
    for (int c0 = 0; c0 < N; c0 += 16) {
      uint32_t v[16];
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
          "%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(dtmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (row_ok)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = t0 + c0 + i;
          if (t < T) Y[(size_t)t * R + row] = __uint_as_float(v[i]) * down;
        }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(dtmem), "r"(kCols) : "memory");
  }
}

template <int N>
static cudaError_t launch_tc5(const uint8_t* W, const float* S, const __half* xh, const __half* xl, float* Y, int R,
                              int K, int T, cudaStream_t st) {
  constexpr size_t sm = (size_t)kTc5Stages * (2 * kTc5ABytes + 2 * N * 32 * 2);
  static bool init = false;  // the attribute is per function; set once per process
  if (!init) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc5_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return e;
    init = true;
  }
  const dim3 grid((R + kTc5Rows - 1) / kTc5Rows, (T + N - 1) / N);
  gemm_tc5_kernel<N><<<grid, kTc5Threads, sm, st>>>(W, S, xh, xl, Y, R, K, T);
  return cudaGetLastError();
}

// Y[T][R] for K a multiple of 32: token tiles of 128 (16, 32 or 64 for fewer tokens).
cudaError_t launch_gemm_tc5(const uint8_t* W, const float* S, const __half* xh, const __half* xl, float* Y, int R,
                            int K, int T, cudaStream_t st) {
  if (T <= 16) return launch_tc5<16>(W, S, xh, xl, Y, R, K, T, st);
  if (T <= 32) return launch_tc5<32>(W, S, xh, xl, Y, R, K, T, st);
  if (T <= 64) return launch_tc5<64>(W, S, xh, xl, Y, R, K, T, st);
  return launch_tc5<128>(W, S, xh, xl, Y, R, K, T, st);
}

}  // namespace mllm
