#pragma once
// Q4 GEMM tile on the 5th-generation tensor cores (tcgen05.mma, accumulator in tensor memory):
// acc[r][t] = W[r0 + r] . X[t0 + t] with W the PGW Q4 rows (engine/infer.js:88-116 per activation row),
// shared by mllm_gemm_q4 (gemm_tc5.cu) and the batched lm_head + argmax (lwe.cu).
//
// One CTA computes a 128-row x N-token tile with three roles and no CTA-wide barrier inside the K loop.
//   - Eight producer warps walk the Q4 groups (32 columns).  Two threads dequantise each weight row's
//     group into the stage's shared memory, then each arrives on the stage's full mbarrier.
//   - One copy thread brings the stage's activation halves (N tokens x 32 columns, hi and lo) by two
//     bulk copies counted on the same barrier (arrive.expect_tx).
//   - One MMA thread waits for a full stage, issues its MMAs and releases the stage with
//     tcgen05.commit onto its empty mbarrier, which the producers and the copy thread wait for before
//     they refill it S groups later.
//
// Precision.  The group scale is folded into the weights, w = (q - 8) s 2^E.  The per-CTA 2^E puts the
// tile's largest |w| near 2^14, so that the fp16 parts below stay normal.  The scale is split as
// s 2^E = sh + sl, sh its top 8 significant bits.  (q - 8) has at most 3 significant bits, so
// w_hi = (q - 8) sh is exact in fp16; w_lo = (q - 8) fl16(sl) carries the rest, to within 2^-18 |w|.
// The activations are split into fp16 x = x_hi + x_lo with |x_lo| <= 2^-11 |x|.  The accumulator
// takes w_hi x_hi + w_hi x_lo + w_lo x_hi in fp32; the dropped w_lo x_lo term is below 2^-18 of each
// product.  The epilogue scales by 2^-E (exact).
//
// Operand layout in shared memory (K-major, no swizzle, the UMMA canonical interleaved form): an 8-row x
// 16-byte core matrix is 128 contiguous bytes; core matrices along K are kTc5Lbo bytes apart, along
// M / N kTc5Sbo bytes apart, so element (row, k) of a 32-column stage sits at
// (row / 8) kTc5Sbo + (k / 8) kTc5Lbo + (row % 8) 16 + (k % 8) 2.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "device_common.cuh"

namespace mllm {
namespace tc5 {

constexpr int kTc5Rows = 128;    // M: weight rows per CTA
constexpr int kTc5Threads = 256;  // two threads per weight row in the dequantisation
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
// 16 consecutive accumulator columns of this warp's 32 tensor-memory lanes (one row per lane).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&f)[16]) {
  uint32_t v[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) f[i] = __uint_as_float(v[i]);
}

// Byte p of w (columns 2p and 2p + 1 of an 8-column chunk) as the fp16 pair (c0 - 8, 16 (c1 - 8)),
// exactly: the nibbles are placed into the mantissas of 1024 and 1024 + 16 c1 and the offsets removed
// by one packed subtraction.
__device__ __forceinline__ __half2 nib_pair(uint32_t w, uint32_t sel) {
  uint32_t x;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(x) : "r"(w), "r"(sel));  // byte p at bytes 0 and 2
  x = (x & 0x00F0000Fu) | 0x64006400u;
  const __half2 h = *reinterpret_cast<const __half2*>(&x);
  return __hsub2(h, __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6480)));  // 1032, 1152
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok)
               : "r"(bar), "r"(parity)
               : "memory");
  return ok != 0;
}
// Wait for phase `parity` of a CTA mbarrier for at most `limit` ns (the clock is read only once the
// first try has failed); false when the limit ran out.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, uint64_t limit) {
  if (bar_try(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!bar_try(bar, parity))
    if (globaltimer() - t0 > limit) return false;
  return true;
}


// Shared-memory bytes of the S-stage ring of tc5_tile<N, S>.
template <int N, int S>
constexpr size_t tc5_smem_bytes() {
  return (size_t)S * (2 * kTc5ABytes + 2 * N * 64);
}

// What the epilogue of a tile needs: the accumulator's tensor-memory address, the 2^-E scale, and
// whether every wait of the tile finished in time (the same on every thread).
struct Tc5Acc {
  uint32_t dtmem;
  float down;
  bool ok;
};

// One 128-row x N-token tile, run by kTc5Threads + 64 threads (see the top of this file):
// rows r0 .. r0 + 127 of the R x K Q4 matrix (W, Sc) against tokens t0 .. t0 + N - 1 of the tiled
// activation halves xh / xl (T8 8-token blocks; see split_tiled_kernel).  smem holds
// tc5_smem_bytes<N, S>() bytes.  With pdl the copy thread waits for the previous kernel
// (griddepcontrol.wait) before its first activation copy; the weights need no wait.  A wait that runs
// out its limit sets *err and turns ok false.  Every thread must then call tc5_release.
template <int N, int S>
__device__ __forceinline__ Tc5Acc tc5_tile(const uint8_t* __restrict__ W, const float* __restrict__ Sc,
                                           const __half* __restrict__ xh, const __half* __restrict__ xl, int R, int K,
                                           int T8, int r0, int t0, uint8_t* smem, bool pdl, int* err) {
  constexpr int kB = N * 64;  // one fp16 half of a stage's activations
  constexpr int kStage = 2 * kTc5ABytes + 2 * kB;
  __shared__ __align__(8) uint64_t full[S], empty[S], done;
  __shared__ uint32_t tmem_base;
  __shared__ float smax[kTc5Threads / 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool producer = tid < kTc5Threads;
  const int NG = K / 32;
  const int lr = (tid >> 1) & (kTc5Rows - 1), half = tid & 1;  // weight row of the tile, and which 16 columns
  const int row = r0 + lr;
  const bool row_ok = producer && row < R;
  const uint64_t limit = kWaitNs;
  // N <= 128: x_hi and x_lo (adjacent in shared memory, the same 512-byte stride) form one 2N-token B
  // operand, so w_hi (x_hi | x_lo) is one MMA and the epilogue adds column j + N to column j
  constexpr bool kMerge = N <= 128;
  constexpr int kAcc = kMerge ? 2 * N : N;
  constexpr uint32_t kCols = kAcc < 32 ? 32 : kAcc;  // tensor-memory columns (a power of 2 >= 32)
  // activation bytes per stage: the 8-token blocks of this tile that exist (the last may be padding)
  const uint32_t xbytes = (uint32_t)min(N / 8, T8 - t0 / 8) * 512u;

  // ---- tensor memory for the accumulator (warp 0), barriers, the tile's power-of-two weight scale
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      // every producer thread, plus the copy thread's arrival with the copies' byte count
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&full[s])), "r"(kTc5Threads + 1) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[s])) : "memory");
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&done)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  float m = 0.f;
  if (row_ok) {
#pragma unroll 8
    for (int g = half; g < NG; g += 2) m = fmaxf(m, fabsf(__ldg(Sc + (size_t)row * NG + g)));
  }
  m = warp_max(m);
  if (lane == 0 && producer) smax[warp] = m;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t dtmem = tmem_base;
  m = 0.f;
  for (int w = 0; w < kTc5Threads / 32; ++w) m = fmaxf(m, smax[w]);
  int e2 = 0;
  if (m > 0.f) (void)frexpf(8.f * m, &e2);  // 8 m < 2^e2
  const int E = 14 - e2;                      // |w| 2^E < 2^14
  const float up = ldexpf(1.f, E), down = ldexpf(1.f, -E);
  bool ok = true;

  if (producer) {
    const uint8_t* wrow = W + (size_t)row * (K / 2);
    const float* srow = Sc + (size_t)row * NG;
    // this thread's nibbles and scale of the next four groups, requested ahead so that the global-load
    // latency overlaps the groups in between (rows past R hold weight 0)
    uint2 q0, q1, q2, q3;
    float s0, s1, s2, s3;
    auto fetch = [&](int g, uint2& q, float& sc) {
      q = make_uint2(0x88888888u, 0x88888888u);
      sc = 0.f;
      if (row_ok && g < NG) {
        q = __ldg(reinterpret_cast<const uint2*>(wrow + 16 * g + 8 * half));
        sc = __ldg(srow + g);
      }
    };
    fetch(0, q0, s0);
    fetch(1, q1, s1);
    fetch(2, q2, s2);
    fetch(3, q3, s3);
    const int rb = (lr >> 3) * kTc5Sbo + (lr & 7) * 16 + 2 * half * kTc5Lbo;
    for (int g = 0; g < NG; ++g) {
      const int s = g % S;
      // the MMAs that read this stage S groups ago are done
      if (ok && g >= S && !bar_wait(su32(&empty[s]), ((g / S) - 1) & 1, limit)) {
        atomicExch(err, 1);
        ok = false;
      }
      uint8_t* st = smem + (size_t)s * kStage;
      // weights: this thread's half (16 columns) of its row's group g.  The scale is split into
      // sh (its top 8 significant bits) + sl; (q - 8) has at most 3 significant bits, so
      // (q - 8) sh is exact in fp16 (the high half) and (q - 8) fl16(sl) carries the rest.
      const uint2 q = q0;
      const float sc = s0 * up;
      q0 = q1;
      s0 = s1;
      q1 = q2;
      s1 = s2;
      q2 = q3;
      s2 = s3;
      fetch(g + 4, q3, s3);
      const float sh = __uint_as_float(__float_as_uint(sc) & 0xFFFF0000u);
      const float sl = sc - sh;
      const __half2 mh = __floats2half2_rn(sh, sh * 0.0625f), ml = __floats2half2_rn(sl, sl * 0.0625f);
      const uint32_t qw[2] = {q.x, q.y};
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        __half2 hi[4], lo[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const __half2 v = nib_pair(qw[c], (uint32_t)(p | (4 << 4) | (p << 8) | (4 << 12)));
          hi[p] = __hmul2(v, mh);
          lo[p] = __hmul2(v, ml);
        }
        *reinterpret_cast<uint4*>(st + rb + c * kTc5Lbo) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(st + kTc5ABytes + rb + c * kTc5Lbo) = *reinterpret_cast<const uint4*>(lo);
      }
      // make this thread's weight writes visible to the tensor cores and mark them done
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&full[s])) : "memory");
    }
  } else if (warp == kTc5Threads / 32 + 1) {
    // ---- the copy warp: per group, once the stage is free, the activation halves by two bulk copies
    if (lane == 0) {
      if (pdl) asm volatile("griddepcontrol.wait;" ::: "memory");  // the activations come from the previous kernel
      for (int g = 0; g < NG; ++g) {
        const int s = g % S;
        if (ok && g >= S && !bar_wait(su32(&empty[s]), ((g / S) - 1) & 1, limit)) {
          atomicExch(err, 1);
          ok = false;
        }
        const uint32_t full_s = su32(&full[s]), st = su32(smem + (size_t)s * kStage);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full_s), "r"(2u * xbytes)
                     : "memory");
        const size_t src = ((size_t)g * T8 + t0 / 8) * 256;  // in halves
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         st + 2 * kTc5ABytes),
                     "l"(xh + src), "r"(xbytes), "r"(full_s)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         st + 2 * kTc5ABytes + kB),
                     "l"(xl + src), "r"(xbytes), "r"(full_s)
                     : "memory");
      }
    }
  } else if (lane == 0) {
    // ---- the MMA warp: per group, wait until full, issue w_hi x_hi + w_hi x_lo + w_lo x_hi, release
    const uint32_t idesc = idesc_f16(N), idesc2 = idesc_f16(kAcc);
    for (int c = 0; c < NG && ok; ++c) {
      const int s = c % S;
      if (!bar_wait(su32(&full[s]), (c / S) & 1, limit)) {
        atomicExch(err, 1);
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t st = su32(smem + (size_t)s * kStage);
#pragma unroll
      for (int j = 0; j < 2; ++j) {  // two K = 16 steps of the group
        const uint64_t ah = sdesc(st + j * 2 * kTc5Lbo), al = sdesc(st + kTc5ABytes + j * 2 * kTc5Lbo);
        const uint64_t bh = sdesc(st + 2 * kTc5ABytes + j * 2 * kTc5Lbo);
        const uint64_t bl = sdesc(st + 2 * kTc5ABytes + kB + j * 2 * kTc5Lbo);
        if constexpr (kMerge) {
          mma_f16(dtmem, ah, bh, idesc2, (c > 0 || j > 0) ? 1u : 0u);  // columns [0, N): x_hi, [N, 2N): x_lo
          mma_f16(dtmem, al, bh, idesc, 1u);
        } else {
          mma_f16(dtmem, ah, bh, idesc, (c > 0 || j > 0) ? 1u : 0u);
          mma_f16(dtmem, ah, bl, idesc, 1u);
          mma_f16(dtmem, al, bh, idesc, 1u);
        }
      }
      mma_commit(su32(&empty[s]));
    }
    mma_commit(su32(&done));  // arrives once every MMA issued above has finished
  }
  __syncwarp();
  // ---- epilogue: every MMA has finished
  if (!bar_wait(su32(&done), 0, limit)) {
    atomicExch(err, 1);
    ok = false;
  }
  if (tid == kTc5Threads + 32) {
    // no bulk copy of this CTA is left in flight: the last use of each stage has completed (at once,
    // unless the MMA warp stopped early)
    for (int s = 0; s < S && s < NG; ++s) {
      const int gl = s + ((NG - 1 - s) / S) * S;
      if (!bar_wait(su32(&full[s]), (gl / S) & 1, limit)) {
        atomicExch(err, 1);
        ok = false;
      }
    }
  }
  ok = __syncthreads_and(ok);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  return Tc5Acc{dtmem, down, ok};
}

// N <= 128 keeps x_hi and x_lo products in separate column halves of the accumulator.
template <int N>
constexpr bool tc5_merged() {
  return N <= 128;
}

// 16 accumulator columns c0 .. c0 + 15 of this warp's 32 rows (tensor-memory lanes 32 (warp % 4) ..),
// summed over the x_hi / x_lo halves and scaled back by 2^-E.
template <int N>
__device__ __forceinline__ void tc5_cols16(const Tc5Acc& acc, int warp, int c0, float (&v)[16]) {
  const uint32_t lrow = acc.dtmem + ((uint32_t)((warp & 3) * 32) << 16);
  tmem_ld16(lrow + (uint32_t)c0, v);
  if constexpr (tc5_merged<N>()) {
    float u[16];
    tmem_ld16(lrow + (uint32_t)(N + c0), u);
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] += u[i];
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] *= acc.down;
}

// Frees the tile's tensor memory; every thread of the CTA calls it once its epilogue is done.
template <int N>
__device__ __forceinline__ void tc5_release(const Tc5Acc& acc) {
  constexpr int kAcc = tc5_merged<N>() ? 2 * N : N;
  constexpr uint32_t kCols = kAcc < 32 ? 32 : kAcc;
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(acc.dtmem), "r"(kCols) : "memory");
  }
}

}  // namespace tc5
}  // namespace mllm
