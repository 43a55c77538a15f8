#pragma once
// Q4 GEMM tile on the 5th-generation tensor cores (tcgen05.mma, accumulator in tensor memory):
// acc[r][t] = W[r0 + r] . X[t0 + t] with W the PGW Q4 rows (engine/infer.js:88-116 per activation row),
// shared by mllm_gemm_q4 (gemm_tc5.cu), the batched lm_head + argmax and the layer GEMMs of long
// token-batch forwards (lwe.cu).
//
// One CTA computes a 128-row x N-token tile with three roles and no CTA-wide barrier inside the K loop.
//   - Eight producer warps walk the Q4 groups (32 columns).  Two threads dequantise each weight row's
//     group into a stage of shared memory; each warp then arrives once on the stage's full mbarrier.
//   - One copy thread brings the activation halves (N tokens x 32 columns, hi and lo) by two bulk copies
//     per stage, counted on the stage's barrier.
//   - One MMA thread waits for a full stage, issues its MMAs and releases the stage with
//     tcgen05.commit onto its empty mbarrier, which the producers and the copy thread wait for before
//     they refill it.
// tc5_tile_pre is the same tile for matrices expanded at load into these stage images: no producer
// warps, the copy thread brings one image per group and every group's activation halves up front.
//
// Precision.  The group scale is folded into the weights, w = (q - 8) s 2^E.  The per-CTA 2^E puts the
// tile's largest |w| near 2^14, so that the fp16 parts below stay normal.  The scale is split as
// s 2^E = sh + sl, sh its top 8 significant bits.  (q - 8) has at most 3 significant bits, so
// w_hi = (q - 8) sh is exact in fp16; w_lo = (q - 8) fl16(sl) carries the rest, to within 2^-18 |w|.
// The activations are split into fp16 x = x_hi + x_lo with |x_lo| <= 2^-11 |x|.  The accumulator
// takes w_hi x_hi + w_hi x_lo + w_lo x_hi in fp32; the dropped w_lo x_lo term is below 2^-18 of each
// product.  The epilogue scales by 2^-E (exact).
//
// Operand layout in shared memory (K-major, 64-byte swizzle): a row of a 32-column group is 64 bytes,
// 8 rows form a 512-byte atom (kTc5Sbo apart along M / N), and the 16-byte chunk j of row r sits at
// chunk position j ^ ((r / 2) % 4), so that the 8 rows of a core matrix fall into different banks.
// Atoms start on 1024-byte boundaries of the shared window (the swizzle reads address bits 4-8).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "device_common.cuh"

namespace mllm {
namespace tc5 {

constexpr int kTc5Rows = 128;    // M: weight rows per CTA
constexpr int kTc5Threads = 256;  // two threads per weight row in the dequantisation
constexpr int kTc5Sbo = 512;     // bytes between 8-row atoms along M / N (8 rows x 64 bytes)
constexpr int kTc5ABytes = kTc5Rows * 32 * 2;  // one fp16 half of a stage's weights: 8 KB

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor (K-major, 64-byte swizzle, version 1; the leading offset is unused for
// a K extent of one swizzle width and set to 16 bytes).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)((kTc5Sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}
// Byte offset of 16-byte chunk j (columns 8 j .. 8 j + 7 of the group) of row r in a swizzled group.
__host__ __device__ __forceinline__ int sw64_at(int r, int j) {
  return (r >> 3) * kTc5Sbo + (r & 7) * 64 + ((j ^ ((r >> 1) & 3)) << 4);
}
// Tiled activation layout the tile reads (in halves): element (t, k) of a T-token x K-column array,
// T8 = ceil(T / 8).  Group k / 32 holds T8 blocks of 8 tokens; a block is one swizzled 512-byte atom, so
// that a bulk copy of whole blocks lands in shared memory in the operand layout.
__host__ __device__ __forceinline__ size_t tiled_at(int t, int k, int T8) {
  return ((size_t)(k >> 5) * T8 + (t >> 3)) * 256 + (sw64_at(t & 7, (k >> 3) & 3) >> 1) + (k & 7);
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


// Shared-memory bytes of the S-stage ring of tc5_tile<N, S> (+ 1 KB to align the atoms).
template <int N, int S>
constexpr size_t tc5_smem_bytes() {
  return (size_t)S * (2 * kTc5ABytes + 2 * N * 64) + 1024;
}

// Row sources of a tile: tile row lr (0 .. 127) -> its packed Q4 row and scales, false past the matrix.
struct Tc5Linear {  // rows r0 .. r0 + 127 of an R x K matrix
  const uint8_t* W;
  const float* S;
  int R, K, r0;
  __host__ __device__ Tc5Linear at_tile(int tile) const { return Tc5Linear{W, S, R, K, tile * kTc5Rows}; }
  __device__ __forceinline__ bool row(int lr, const uint8_t*& w, const float*& s) const {
    const int r = r0 + lr;
    if (r >= R) return false;
    w = W + (size_t)r * (K / 2);
    s = S + (size_t)r * (K / 32);
    return true;
  }
};
// w1 / w3 pairs of 64 FF rows f0 .. f0 + 63: tile row 32 q + j is w1 row f0 + 16 q + j for j < 16 and
// w3 row f0 + 16 q + j - 16 for j >= 16, so that lanes j and j + 16 of the warp that drains quarter q
// hold the two products of one FF row.
struct Tc5Paired {
  const uint8_t* W1;
  const float* S1;
  const uint8_t* W3;
  const float* S3;
  int F, K, f0;
  __host__ __device__ Tc5Paired at_tile(int tile) const { return Tc5Paired{W1, S1, W3, S3, F, K, tile * 64}; }
  __device__ __forceinline__ bool row(int lr, const uint8_t*& w, const float*& s) const {
    const int j = lr & 31, f = f0 + 16 * (lr >> 5) + (j & 15);
    if (f >= F) return false;
    w = (j < 16 ? W1 : W3) + (size_t)f * (K / 2);
    s = (j < 16 ? S1 : S3) + (size_t)f * (K / 32);
    return true;
  }
};

// What the epilogue of a tile needs: the accumulator's tensor-memory address, the 2^-E scale, and
// whether every wait of the tile finished in time (the same on every thread).
struct Tc5Acc {
  uint32_t dtmem;
  float down;
  bool ok;
};
struct Tc5NoSide {
  __device__ __forceinline__ void operator()(int) const {}
};

// One 128-row x N-token tile over the Q4 groups g0 .. g0 + ng - 1, run by kTc5Threads + 64 threads
// (see the top of this file): the tile rows of `rows` against tokens t0 .. t0 + N - 1 of the tiled
// activation halves xh / xl (T8 8-token blocks, tiled_at), through S one-group stages of weights and
// activations (tc5_smem_bytes<N, S>()); each producer thread fetches its nibbles and scales kPD groups
// ahead into registers.  With pdl the copy thread waits for the previous kernel (griddepcontrol.wait)
// before its first activation copy; the weights need no wait.  Lanes 1 .. 31 of the copy warp run
// side(lane) during the K loop (after the same wait when pdl): epilogue inputs that the previous kernel
// wrote can be staged there.  A wait that runs out its limit sets *err and turns ok false.  Every thread
// must then call tc5_release.
template <int N, int S, class Rows, class Side = Tc5NoSide>
__device__ __forceinline__ Tc5Acc tc5_tile_rows(const Rows& rows, const __half* __restrict__ xh,
                                                const __half* __restrict__ xl, int T8, int t0, int g0, int ng,
                                                uint8_t* smem, bool pdl, int* err, const Side& side = Tc5NoSide{}) {
  constexpr int kB = N * 64;                    // one fp16 half of a group's activations
  constexpr int kPD = 8;                        // groups each producer thread requests ahead
  constexpr int kStageA = 2 * kTc5ABytes;       // a stage's weights: [w_hi 8 KB][w_lo 8 KB]
  __shared__ __align__(8) uint64_t full[S], empty[S], done;
  __shared__ uint32_t tmem_base;
  __shared__ float smax[kTc5Threads / 32];
  smem += (1024u - (su32(smem) & 1023u)) & 1023u;  // swizzle atoms on 1024-byte boundaries
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool producer = tid < kTc5Threads;
  const int lr = (tid >> 1) & (kTc5Rows - 1), half = tid & 1;  // weight row of the tile, and which 16 columns
  const uint8_t* wrow = nullptr;
  const float* srow = nullptr;
  const bool row_ok = producer && rows.row(lr, wrow, srow);
  const uint64_t limit = kWaitNs;
  // N <= 128: x_hi and x_lo (adjacent in shared memory, the same 512-byte stride) form one 2N-token B
  // operand, so w_hi (x_hi | x_lo) is one MMA and the epilogue adds column j + N to column j
  constexpr bool kMerge = N <= 128;
  constexpr int kAcc = kMerge ? 2 * N : N;
  constexpr uint32_t kCols = kAcc < 32 ? 32 : kAcc;  // tensor-memory columns (a power of 2 >= 32)
  // activation bytes per group: the 8-token blocks of this tile that exist (the last may be padding)
  const uint32_t xbytes = (uint32_t)min(N / 8, T8 - t0 / 8) * 512u;
  uint8_t* const xs = smem + (size_t)S * kStageA;  // activations: S ring stages

  // ---- tensor memory for the accumulator (warp 0), barriers, the tile's power-of-two weight scale
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      // one arrival per producer warp, plus the copy thread's arrival with the copies' bytes
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&full[s])), "r"(kTc5Threads / 32 + 1)
                   : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[s])) : "memory");
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&done)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // this thread's nibbles and scales of the first kPD groups, requested before the scale
  // pass so that both round trips overlap (volatile loads: issued where written)
  uint2 q[kPD];
  float sc[kPD];
  auto fetch = [&](int c, uint2& qq, float& ss) {
    qq = make_uint2(0x88888888u, 0x88888888u);
    ss = 0.f;
    if (row_ok && c < ng) {
      const uint8_t* p = wrow + 16 * (g0 + c) + 8 * half;
      asm volatile("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(qq.x), "=r"(qq.y) : "l"(p));
      ss = ldv_f32(srow + g0 + c);
    }
  };
  float m = 0.f;
  if (producer) {
#pragma unroll
    for (int i = 0; i < kPD; ++i) fetch(i, q[i], sc[i]);
  }
  if (row_ok) {
#pragma unroll 8
    for (int g = half; g < ng; g += 2) m = fmaxf(m, fabsf(__ldg(srow + g0 + g)));
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
    const int rb0 = sw64_at(lr, 2 * half), rb1 = sw64_at(lr, 2 * half + 1);  // this thread's two chunks
    // weights: this thread's half (16 columns) of its row's group.  The scale is split into
    // sh (its top 8 significant bits) + sl; (q - 8) has at most 3 significant bits, so
    // (q - 8) sh is exact in fp16 (the high half) and (q - 8) fl16(sl) carries the rest.
    auto dequant = [&](uint8_t* st, uint2 qc, float scale) {
      const float sh = __uint_as_float(__float_as_uint(scale) & 0xFFFF0000u);
      const float sl = scale - sh;
      const __half2 mh = __floats2half2_rn(sh, sh * 0.0625f), ml = __floats2half2_rn(sl, sl * 0.0625f);
      const uint32_t qw[2] = {qc.x, qc.y};
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        __half2 hi[4], lo[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const __half2 v = nib_pair(qw[cc], (uint32_t)(p | (4 << 4) | (p << 8) | (4 << 12)));
          hi[p] = __hmul2(v, mh);
          lo[p] = __hmul2(v, ml);
        }
        const int rb = cc ? rb1 : rb0;
        *reinterpret_cast<uint4*>(st + rb) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(st + kTc5ABytes + rb) = *reinterpret_cast<const uint4*>(lo);
      }
    };
    // the MMAs that read stage s one round ago are done (one lane waits for the warp)
    auto stage_free = [&](int k, int s) {
      if (k >= S) {
        if (lane == 0 && ok && !bar_wait(su32(&empty[s]), ((k / S) - 1) & 1, limit)) {
          atomicExch(err, 1);
          ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
    };
    // make the warp's weight writes visible to the tensor cores, then one arrival for the warp
    auto stage_full = [&](int s) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&full[s])) : "memory");
    };
    // the nibbles and scales of group c + kPD are requested while group c is dequantised, so that the
    // global-load latency overlaps the groups in between (rows past the matrix hold weight 0)
    for (int cb = 0; cb < ng; cb += kPD) {
#pragma unroll
      for (int i = 0; i < kPD; ++i) {
        const int c = cb + i;
        if (c >= ng) break;
        const int s = c % S;
        stage_free(c, s);
        const uint2 qc = q[i];
        const float scale = sc[i] * up;
        fetch(c + kPD, q[i], sc[i]);
        dequant(smem + (size_t)s * kStageA, qc, scale);
        stage_full(s);
      }
    }
  } else if (warp == kTc5Threads / 32 + 1) {
    // ---- the copy warp: the activation halves of each group by two bulk copies
    if (lane != 0) {
      if (pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
      side(lane);
    } else {
      if (pdl) asm volatile("griddepcontrol.wait;" ::: "memory");  // the activations come from the previous kernel
      for (int c = 0; c < ng; ++c) {
        // a ring: wait until the MMAs of S groups ago released the stage
        const int s = c % S;
        if (ok && c >= S && !bar_wait(su32(&empty[s]), ((c / S) - 1) & 1, limit)) {
          atomicExch(err, 1);
          ok = false;
        }
        const uint32_t bar = su32(&full[s]), dst = su32(xs + (size_t)s * 2 * kB);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(2u * xbytes) : "memory");
        const size_t src = ((size_t)(g0 + c) * T8 + t0 / 8) * 256;  // in halves
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst),
                     "l"(xh + src), "r"(xbytes), "r"(bar)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst + kB),
                     "l"(xl + src), "r"(xbytes), "r"(bar)
                     : "memory");
      }
    }
  } else if (lane == 0) {
    // ---- the MMA warp: per group, wait until full, issue w_hi x_hi + w_hi x_lo + w_lo x_hi, release
    const uint32_t idesc = idesc_f16(N), idesc2 = idesc_f16(kAcc);
    for (int c = 0; c < ng && ok; ++c) {
      const int s = c % S;
      if (!bar_wait(su32(&full[s]), (c / S) & 1, limit)) {
        atomicExch(err, 1);
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t st = su32(smem + (size_t)s * kStageA);
      const uint32_t xb = su32(xs + (size_t)s * 2 * kB);
#pragma unroll
      for (int j = 0; j < 2; ++j) {  // two K = 16 steps of the group: 32 bytes into each 64-byte row
        const uint64_t ah = sdesc(st + j * 32), al = sdesc(st + kTc5ABytes + j * 32);
        const uint64_t bh = sdesc(xb + j * 32);
        const uint64_t bl = sdesc(xb + kB + j * 32);
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
  // ---- epilogue: every MMA has finished (one lane per warp waits)
  if (lane == 0 && !bar_wait(su32(&done), 0, limit)) {
    atomicExch(err, 1);
    ok = false;
  }
  if (tid == kTc5Threads + 32) {
    // no bulk copy of this CTA is left in flight (at once, unless a wait above ran out)
    for (int s = 0; s < S && s < ng; ++s) {  // the last use of each stage
      const int gl = s + ((ng - 1 - s) / S) * S;
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

// ---- Pre-expanded weights.  tc5_expand_kernel writes, once at load, every (128-row tile, group) of a Q4
// matrix as the exact shared-memory image the producers would build: [w_hi 8 KB][w_lo 8 KB] in the
// swizzled layout, with the tile's 2^E factor applied (E from the largest |scale| of the tile's rows over
// all groups), and the tile's 2^-E in `down`.  The values equal those of tc5_tile_rows (whose E spans the
// CTA's groups only), so a tile computes the same products, now fed by one bulk copy per group.
constexpr int kTc5GroupImage = 2 * kTc5ABytes;  // bytes of one (tile, group) image
template <class Rows>
__global__ void __launch_bounds__(256) tc5_expand_kernel(Rows rows, int NG, uint8_t* __restrict__ out,
                                                         float* __restrict__ down) {
  __shared__ float smax[8];
  const int tile = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lr = tid >> 1, half = tid & 1;
  const uint8_t* wrow = nullptr;
  const float* srow = nullptr;
  const bool ok = rows.at_tile(tile).row(lr, wrow, srow);
  float m = 0.f;
  if (ok)
    for (int k = half; k < NG; k += 2) m = fmaxf(m, fabsf(srow[k]));
  m = warp_max(m);
  if ((tid & 31) == 0) smax[tid >> 5] = m;
  __syncthreads();
  m = 0.f;
  for (int w = 0; w < 8; ++w) m = fmaxf(m, smax[w]);
  int e2 = 0;
  if (m > 0.f) (void)frexpf(8.f * m, &e2);
  const int E = 14 - e2;
  const float up = ldexpf(1.f, E);
  if (g == 0 && tid == 0) down[tile] = ldexpf(1.f, -E);
  uint2 q = make_uint2(0x88888888u, 0x88888888u);
  float scale = 0.f;
  if (ok) {
    q = *reinterpret_cast<const uint2*>(wrow + 16 * g + 8 * half);
    scale = srow[g] * up;
  }
  const float sh = __uint_as_float(__float_as_uint(scale) & 0xFFFF0000u), sl = scale - sh;
  const __half2 mh = __floats2half2_rn(sh, sh * 0.0625f), ml = __floats2half2_rn(sl, sl * 0.0625f);
  uint8_t* img = out + ((size_t)tile * NG + g) * kTc5GroupImage;
  const uint32_t qw[2] = {q.x, q.y};
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    __half2 hi[4], lo[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __half2 v = nib_pair(qw[cc], (uint32_t)(p | (4 << 4) | (p << 8) | (4 << 12)));
      hi[p] = __hmul2(v, mh);
      lo[p] = __hmul2(v, ml);
    }
    const int rb = sw64_at(lr, 2 * half + cc);
    *reinterpret_cast<uint4*>(img + rb) = *reinterpret_cast<const uint4*>(hi);
    *reinterpret_cast<uint4*>(img + kTc5ABytes + rb) = *reinterpret_cast<const uint4*>(lo);
  }
}

// Shared-memory bytes of tc5_tile_pre<N, S> over ng groups: S group images and every group's
// activation halves.
__host__ __device__ constexpr size_t tc5_smem_pre(int N, int S, int ng) {
  return (size_t)S * kTc5GroupImage + (size_t)ng * 2 * N * 64 + 1024;
}

// One 128-row x N-token tile over groups g0 .. g0 + ng - 1 of a pre-expanded matrix: img points at the
// tile's first group image, down is its 2^-E.  No producer warps: the copy thread brings the group images
// through an S-stage ring (the first S before the wait for the previous kernel, which the weights do not
// need) and every group's activation halves at once; the MMA thread is the one of tc5_tile_rows.  Lanes
// 1 .. 31 of the copy warp run side(lane) as there.  Waits are bounded; every thread must then call
// tc5_release.
template <int N, int S, class Side = Tc5NoSide>
__device__ __forceinline__ Tc5Acc tc5_tile_pre(const uint8_t* __restrict__ img, float down,
                                               const __half* __restrict__ xh, const __half* __restrict__ xl, int T8,
                                               int t0, int g0, int ng, uint8_t* smem, bool pdl, int* err,
                                               const Side& side = Tc5NoSide{}) {
  constexpr int kB = N * 64;
  __shared__ __align__(8) uint64_t full[S], empty[S], done, xfull;
  __shared__ uint32_t tmem_base;
  smem += (1024u - (su32(smem) & 1023u)) & 1023u;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t limit = kWaitNs;
  constexpr bool kMerge = N <= 128;
  constexpr int kAcc = kMerge ? 2 * N : N;
  constexpr uint32_t kCols = kAcc < 32 ? 32 : kAcc;
  const uint32_t xbytes = (uint32_t)min(N / 8, T8 - t0 / 8) * 512u;
  uint8_t* const xs = smem + (size_t)S * kTc5GroupImage;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&full[s])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&empty[s])) : "memory");
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&done)) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&xfull)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t dtmem = tmem_base;
  bool ok = true;
  auto load_image = [&](int c) {
    const uint32_t bar = su32(&full[c % S]);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)kTc5GroupImage)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     su32(smem + (size_t)(c % S) * kTc5GroupImage)),
                 "l"(img + (size_t)c * kTc5GroupImage), "r"((uint32_t)kTc5GroupImage), "r"(bar)
                 : "memory");
  };
  if (warp == kTc5Threads / 32 + 1) {
    if (lane != 0) {
      if (pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
      side(lane);
    } else {
      for (int c = 0; c < ng && c < S; ++c) load_image(c);  // weights: no wait for the previous kernel
      if (pdl) asm volatile("griddepcontrol.wait;" ::: "memory");
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&xfull)),
                   "r"(2u * xbytes * (uint32_t)ng)
                   : "memory");
      for (int c = 0; c < ng; ++c) {
        const size_t src = ((size_t)(g0 + c) * T8 + t0 / 8) * 256;  // in halves
        const uint32_t dst = su32(xs + (size_t)c * 2 * kB), bar = su32(&xfull);
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst),
                     "l"(xh + src), "r"(xbytes), "r"(bar)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst + kB),
                     "l"(xl + src), "r"(xbytes), "r"(bar)
                     : "memory");
      }
      for (int c = S; c < ng; ++c) {  // the ring: a stage is refilled once its MMAs are done
        if (!bar_wait(su32(&empty[c % S]), ((c / S) - 1) & 1, limit)) {
          atomicExch(err, 1);
          ok = false;
          break;
        }
        load_image(c);
      }
    }
  } else if (warp == kTc5Threads / 32 && lane == 0) {
    const uint32_t idesc = idesc_f16(N), idesc2 = idesc_f16(kAcc);
    if (!bar_wait(su32(&xfull), 0, limit)) {
      atomicExch(err, 1);
      ok = false;
    }
    for (int c = 0; c < ng && ok; ++c) {
      const int s = c % S;
      if (!bar_wait(su32(&full[s]), (c / S) & 1, limit)) {
        atomicExch(err, 1);
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t st = su32(smem + (size_t)s * kTc5GroupImage);
      const uint32_t xb = su32(xs + (size_t)c * 2 * kB);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint64_t ah = sdesc(st + j * 32), al = sdesc(st + kTc5ABytes + j * 32);
        const uint64_t bh = sdesc(xb + j * 32);
        const uint64_t bl = sdesc(xb + kB + j * 32);
        if constexpr (kMerge) {
          mma_f16(dtmem, ah, bh, idesc2, (c > 0 || j > 0) ? 1u : 0u);
          mma_f16(dtmem, al, bh, idesc, 1u);
        } else {
          mma_f16(dtmem, ah, bh, idesc, (c > 0 || j > 0) ? 1u : 0u);
          mma_f16(dtmem, ah, bl, idesc, 1u);
          mma_f16(dtmem, al, bh, idesc, 1u);
        }
      }
      mma_commit(su32(&empty[s]));
    }
    mma_commit(su32(&done));
  }
  __syncwarp();
  if (lane == 0 && !bar_wait(su32(&done), 0, limit)) {
    atomicExch(err, 1);
    ok = false;
  }
  if (tid == kTc5Threads + 32) {  // no bulk copy of this CTA is left in flight
    if (!bar_wait(su32(&xfull), 0, limit)) {
      atomicExch(err, 1);
      ok = false;
    }
    for (int s = 0; s < S && s < ng; ++s) {  // the last image copied into each stage
      const int gl = s + ((ng - 1 - s) / S) * S;
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

// The whole K range of rows r0 .. r0 + 127 of an R x K matrix, activations in the ring form.
template <int N, int S>
__device__ __forceinline__ Tc5Acc tc5_tile(const uint8_t* __restrict__ W, const float* __restrict__ Sc,
                                           const __half* __restrict__ xh, const __half* __restrict__ xl, int R, int K,
                                           int T8, int r0, int t0, uint8_t* smem, bool pdl, int* err) {
  return tc5_tile_rows<N, S>(Tc5Linear{W, Sc, R, K, r0}, xh, xl, T8, t0, 0, K / 32, smem, pdl, err);
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
