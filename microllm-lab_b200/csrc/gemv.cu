// Standalone Q4 group-32 GEMV / skinny GEMM (M <= 16 activation rows) on CUDA cores:
// y[m][r] = sum_g sc[r][g] * sum_k (q[r][32g+k] - 8) * x[m][32g+k]   (engine/infer.js:88-116).
//
// Streaming design: each warp owns ROWS consecutive rows; every lane issues all of its 4-byte weight
// loads (and scale loads) for those rows before the first FMA, so a CTA keeps
// 8 warps x ROWS x cols/2 bytes in flight.  Activations are read through the read-only cache (they
// are small and shared by every row).  fp32 accumulation.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "../../include/mllm.h"
#include "device_common.cuh"
#include "q4mma.cuh"

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

// ---------------------------------------------------------------------------------------------
// Tensor-core GEMV for few activation rows (M <= 16).  A warp owns a 16-row weight tile; per 32-wide
// group each lane loads the 16 packed bytes of rows gid and gid + 8 (one 128-bit load each), turns
// them into fp16 A fragments in registers (exact small integers, nib_pair_f16) and issues one
// mma.m16n8k16 per 16-k block and pass.  The 8 B columns of a pass carry 4 tokens x (fp16 hi, fp16
// lo) of the activations, so lane (gid, t) ends with row gid / gid + 8 of token 4p + t as d0 + d1 and
// d2 + d3, scaled by the group scale in fp32.  The B fragments of all passes are built once per CTA
// in shared memory.  Compared with the CUDA-core kernel this replaces ~9 instructions per weight
// element (dequant, convert, FMA) by ~2.5.  KSL warps may split the k groups of one tile (small R).
// ---------------------------------------------------------------------------------------------
template <int NP, int KSL>
__global__ void __launch_bounds__(256) gemv_q4_tc_kernel(const uint8_t* __restrict__ W, const float* __restrict__ S,
                                                         const float* __restrict__ X, float* __restrict__ Y, int R,
                                                         int K, int M) {
  extern __shared__ __align__(16) uint2 bfrag[];  // [NP][nkb][32]
  __shared__ float red[8][NP][2][32];
  const int nkb = K >> 4, ng = K >> 5, half_k = K >> 1;
  // B fragments: lane (gid, t) of pass p holds column gid = token 4p + gid/2, part gid&1 (hi, lo), at
  // k = 16 kb + 2t, +1 (b0) and + 8, + 9 (b1)
  for (int e = threadIdx.x; e < NP * nkb * 32; e += blockDim.x) {
    const int lane = e & 31, kb = (e >> 5) % nkb, p = e / (32 * nkb);
    const int gid = lane >> 2, t = lane & 3, m = 4 * p + (gid >> 1), part = gid & 1;
    const int k0 = kb * 16 + 2 * t;
    __half v[4];
    const int ks[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half hi = __float2half_rn(0.f), lo = hi;
      if (m < M) split_hi_lo(X[(size_t)m * K + ks[j]], hi, lo);
      v[j] = part ? lo : hi;
    }
    const __half2 b0 = __halves2half2(v[0], v[1]), b1 = __halves2half2(v[2], v[3]);
    bfrag[e] = make_uint2(*reinterpret_cast<const uint32_t*>(&b0), *reinterpret_cast<const uint32_t*>(&b1));
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  constexpr int kTilesPerCta = 8 / KSL;
  const int ntiles = (R + 15) >> 4;
  const int ksl = warp % KSL;
  for (int tile0 = blockIdx.x * kTilesPerCta; tile0 < ntiles; tile0 += gridDim.x * kTilesPerCta) {
    const int tile = tile0 + warp / KSL;
    const int r0 = tile * 16;
    const int ra = min(r0 + gid, R - 1), rb = min(r0 + gid + 8, R - 1);
    const uint8_t* wa = W + (size_t)ra * half_k;
    const uint8_t* wb = W + (size_t)rb * half_k;
    const float* sa = S + (size_t)ra * ng;
    const float* sb = S + (size_t)rb * ng;
    float acc[NP][2];
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[p][0] = acc[p][1] = 0.f;
    if (tile < ntiles) {
      // groups ksl, ksl + KSL, ...; loads run kPre groups ahead
      constexpr int kPre = 4;
      uint4 qa[kPre], qb[kPre];
      float fa[kPre], fb[kPre];
#pragma unroll
      for (int i = 0; i < kPre; ++i) {
        const int g = ksl + i * KSL;
        if (g < ng) {
          qa[i] = __ldg(reinterpret_cast<const uint4*>(wa + g * 16));
          qb[i] = __ldg(reinterpret_cast<const uint4*>(wb + g * 16));
          fa[i] = __ldg(sa + g);
          fb[i] = __ldg(sb + g);
        }
      }
      for (int i0 = 0; ksl + i0 * KSL < ng; i0 += kPre) {
#pragma unroll
        for (int i = 0; i < kPre; ++i) {
          const int g = ksl + (i0 + i) * KSL;
          if (g >= ng) break;
          uint32_t a0[4], a1[4];
          a0[0] = nib_pair_f16(qa[i].x, t);
          a0[1] = nib_pair_f16(qb[i].x, t);
          a0[2] = nib_pair_f16(qa[i].y, t);
          a0[3] = nib_pair_f16(qb[i].y, t);
          a1[0] = nib_pair_f16(qa[i].z, t);
          a1[1] = nib_pair_f16(qb[i].z, t);
          a1[2] = nib_pair_f16(qa[i].w, t);
          a1[3] = nib_pair_f16(qb[i].w, t);
          const float s0 = fa[i], s1 = fb[i];
          const int gn = g + kPre * KSL;  // refill this slot
          if (gn < ng) {
            qa[i] = __ldg(reinterpret_cast<const uint4*>(wa + gn * 16));
            qb[i] = __ldg(reinterpret_cast<const uint4*>(wb + gn * 16));
            fa[i] = __ldg(sa + gn);
            fb[i] = __ldg(sb + gn);
          }
#pragma unroll
          for (int p = 0; p < NP; ++p) {
            const uint2 b0 = bfrag[((size_t)p * nkb + 2 * g) * 32 + lane];
            const uint2 b1 = bfrag[((size_t)p * nkb + 2 * g + 1) * 32 + lane];
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(d, a0, b0.x, b0.y);
            mma16816(d, a1, b1.x, b1.y);
            acc[p][0] = fmaf(s0, d[0] + d[1], acc[p][0]);
            acc[p][1] = fmaf(s1, d[2] + d[3], acc[p][1]);
          }
        }
      }
    }
    if (KSL > 1) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        red[warp][p][0][lane] = acc[p][0];
        red[warp][p][1][lane] = acc[p][1];
      }
      __syncthreads();
      if (ksl == 0) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
          for (int w = 1; w < KSL; ++w) {
            acc[p][0] += red[warp + w][p][0][lane];
            acc[p][1] += red[warp + w][p][1][lane];
          }
      }
      __syncthreads();
    }
    if (ksl == 0 && tile < ntiles) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        const int m = 4 * p + t;
        if (m < M) {
          if (r0 + gid < R) Y[(size_t)m * R + r0 + gid] = acc[p][0];
          if (r0 + gid + 8 < R) Y[(size_t)m * R + r0 + gid + 8] = acc[p][1];
        }
      }
    }
  }
}

// Streaming form for many rows (R >= 1024, K <= 1024): the CTA walks its rows 128 at a time (8 tiles
// of 16 rows, one per warp); a stage = the 128 rows' packed bytes and scales, which are contiguous in
// the PGW layout, brought into shared memory by two bulk copies (cp.async.bulk, completion on an
// mbarrier) kNS stages ahead, so each SM keeps ~100 KB of weights in flight without registers.  A
// partial last stage is read with plain loads.  Waits are bounded (error flag, no hang).
constexpr int kBulkRows = 128;
constexpr int kBulkNS = 3;

// KSL warps share each 16-row tile (k groups interleaved) for more warps in flight per SM.
template <int NP, int KSL, int NSB = kBulkNS, int MINB = 1>
__global__ void __launch_bounds__(256 * KSL, MINB) gemv_q4_bulk_kernel(const uint8_t* __restrict__ W,
                                                                    const float* __restrict__ S,
                                                                    const float* __restrict__ X,
                                                                    float* __restrict__ Y, int R, int K, int M,
                                                                    int* err) {
  __shared__ float red[8 * KSL][NP][2][32];
  extern __shared__ __align__(128) unsigned char sm[];
  const int nkb = K >> 4, ng = K >> 5, half_k = K >> 1;
  const size_t wbytes = (size_t)kBulkRows * half_k, sbytes = (size_t)kBulkRows * ng * 4;
  const size_t stage_bytes = (wbytes + sbytes + 127) & ~(size_t)127;
  uint2* bfrag = reinterpret_cast<uint2*>(sm + NSB * stage_bytes);  // [NP][nkb][32]
  __shared__ __align__(8) uint64_t full[NSB];
  const int nstage_total = (R + kBulkRows - 1) / kBulkRows;
  // this CTA's stages: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_n = nstage_total > (int)blockIdx.x ? (nstage_total - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  auto stage_rows = [&](int j) { return min(kBulkRows, R - ((int)blockIdx.x + j * (int)gridDim.x) * kBulkRows); };
  auto issue = [&](int j) {  // thread 0: bulk copies of stage j (full stages only)
    const int r0 = ((int)blockIdx.x + j * (int)gridDim.x) * kBulkRows;
    unsigned char* dst = sm + (j % NSB) * stage_bytes;
    uint64_t* bar = &full[j % NSB];
    mbar_expect_tx(bar, (uint32_t)(wbytes + sbytes));
    bulk_g2s(dst, W + (size_t)r0 * half_k, (uint32_t)wbytes, bar);
    bulk_g2s(dst + wbytes, S + (size_t)r0 * ng, (uint32_t)sbytes, bar);
  };
  if (threadIdx.x == 0) {
    for (int i = 0; i < NSB; ++i) mbar_init(&full[i], 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int j = 0; j < NSB && j < my_n; ++j)
      if (stage_rows(j) == kBulkRows) issue(j);
  // B fragments (as in the register-prefetch kernel) while the first stages are in flight
  for (int e = threadIdx.x; e < NP * nkb * 32; e += blockDim.x) {
    const int lane = e & 31, kb = (e >> 5) % nkb, p = e / (32 * nkb);
    const int gid = lane >> 2, t = lane & 3, m = 4 * p + (gid >> 1), part = gid & 1;
    const int k0 = kb * 16 + 2 * t;
    __half v[4];
    const int ks[4] = {k0, k0 + 1, k0 + 8, k0 + 9};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      __half hi = __float2half_rn(0.f), lo = hi;
      if (m < M) split_hi_lo(X[(size_t)m * K + ks[q]], hi, lo);
      v[q] = part ? lo : hi;
    }
    const __half2 b0 = __halves2half2(v[0], v[1]), b1 = __halves2half2(v[2], v[3]);
    bfrag[e] = make_uint2(*reinterpret_cast<const uint32_t*>(&b0), *reinterpret_cast<const uint32_t*>(&b1));
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int warp = wid / KSL, ksl = wid % KSL;  // tile of the stage, share of its k groups
  bool ok = true;
  for (int j = 0; j < my_n; ++j) {
    const int r0 = ((int)blockIdx.x + j * (int)gridDim.x) * kBulkRows;
    const int nr = stage_rows(j);
    unsigned char* st = sm + (j % NSB) * stage_bytes;
    if (nr == kBulkRows) {
      if (!mbar_wait_bounded(&full[j % NSB], (uint32_t)((j / NSB) & 1), kWaitNs)) {
        if (threadIdx.x == 0) atomicExch(err, 1);
        mbar_wait_bounded(&full[j % NSB], (uint32_t)((j / NSB) & 1), kWaitNs);
        ok = false;
      }
    } else {  // partial last stage: plain loads
      for (size_t i = threadIdx.x; i < (size_t)nr * half_k / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(st)[i] = reinterpret_cast<const uint32_t*>(W + (size_t)r0 * half_k)[i];
      for (size_t i = threadIdx.x; i < (size_t)nr * ng; i += blockDim.x)
        reinterpret_cast<float*>(st + wbytes)[i] = S[(size_t)r0 * ng + i];
    }
    __syncthreads();  // stage (and, the first time, the B fragments) visible to every warp
    const int tr = warp * 16;  // this warp's tile inside the stage
    const int la = min(tr + gid, nr - 1), lb = min(tr + gid + 8, nr - 1);
    const uint8_t* wa = st + (size_t)la * half_k;
    const uint8_t* wb = st + (size_t)lb * half_k;
    const float* sa = reinterpret_cast<const float*>(st + wbytes) + (size_t)la * ng;
    const float* sb = reinterpret_cast<const float*>(st + wbytes) + (size_t)lb * ng;
    float acc[NP][2];
#pragma unroll
    for (int p = 0; p < NP; ++p) acc[p][0] = acc[p][1] = 0.f;
    if (tr < nr) {
#pragma unroll 3
      for (int g = ksl; g < ng; g += KSL) {  // independent groups: unrolled for overlapping mma chains
        const uint4 qa = *reinterpret_cast<const uint4*>(wa + g * 16);
        const uint4 qb = *reinterpret_cast<const uint4*>(wb + g * 16);
        uint32_t a0[4], a1[4];
        a0[0] = nib_pair_f16(qa.x, t);
        a0[1] = nib_pair_f16(qb.x, t);
        a0[2] = nib_pair_f16(qa.y, t);
        a0[3] = nib_pair_f16(qb.y, t);
        a1[0] = nib_pair_f16(qa.z, t);
        a1[1] = nib_pair_f16(qb.z, t);
        a1[2] = nib_pair_f16(qa.w, t);
        a1[3] = nib_pair_f16(qb.w, t);
        const float s0 = sa[g], s1 = sb[g];
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const uint2 b0 = bfrag[((size_t)p * nkb + 2 * g) * 32 + lane];
          const uint2 b1 = bfrag[((size_t)p * nkb + 2 * g + 1) * 32 + lane];
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma16816(d, a0, b0.x, b0.y);
          mma16816(d, a1, b1.x, b1.y);
          acc[p][0] = fmaf(s0, d[0] + d[1], acc[p][0]);
          acc[p][1] = fmaf(s1, d[2] + d[3], acc[p][1]);
        }
      }
    }
    if (KSL > 1) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        red[wid][p][0][lane] = acc[p][0];
        red[wid][p][1][lane] = acc[p][1];
      }
    }
    __syncthreads();  // every warp is done with this stage's buffer (and its partial sums are out)
    if (ok && ksl == 0 && tr < nr) {
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        for (int w = 1; w < KSL; ++w) {
          acc[p][0] += red[wid + w][p][0][lane];
          acc[p][1] += red[wid + w][p][1][lane];
        }
        const int m = 4 * p + t;
        if (m < M) {
          if (tr + gid < nr) Y[(size_t)m * R + r0 + tr + gid] = acc[p][0];
          if (tr + gid + 8 < nr) Y[(size_t)m * R + r0 + tr + gid + 8] = acc[p][1];
        }
      }
    }
    if (KSL > 1) __syncthreads();  // red is reused by the next stage
    if (threadIdx.x == 0 && j + NSB < my_n && stage_rows(j + NSB) == kBulkRows) issue(j + NSB);
  }
}

template <int NP, int KSL = 2, int NSB = kBulkNS, int MINB = 1>
static cudaError_t run_gemv_bulk(const uint8_t* W, const float* S, const float* X, float* Y, int R, int K, int M,
                                 int* err, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t wbytes = (size_t)kBulkRows * (K / 2), sbytes = (size_t)kBulkRows * (K / 32) * 4;
  const size_t stage_bytes = (wbytes + sbytes + 127) & ~(size_t)127;
  const size_t smem = NSB * stage_bytes + (size_t)NP * (K / 16) * 32 * sizeof(uint2);
  const cudaError_t e = cudaFuncSetAttribute(gemv_q4_bulk_kernel<NP, KSL, NSB, MINB>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int nst = (R + kBulkRows - 1) / kBulkRows;
  gemv_q4_bulk_kernel<NP, KSL, NSB, MINB><<<std::min(nst, MINB * sms), 256 * KSL, smem, st>>>(W, S, X, Y, R, K, M, err);
  return cudaGetLastError();
}

constexpr size_t kBulk2Smem = 108 * 1024;  // dynamic shared memory of a CTA when two share an SM
static size_t gemv_bulk_smem(int K, int np, int ns = kBulkNS) {
  const size_t wbytes = (size_t)kBulkRows * (K / 2), sbytes = (size_t)kBulkRows * (K / 32) * 4;
  return ns * ((wbytes + sbytes + 127) & ~(size_t)127) + (size_t)np * (K / 16) * 32 * 8;
}

template <int NP, int KSL>
static cudaError_t run_gemv_tc(const uint8_t* W, const float* S, const float* X, float* Y, int R, int K, int M,
                               cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = (size_t)NP * (K >> 4) * 32 * sizeof(uint2);
  const size_t static_smem = (size_t)8 * NP * 2 * 32 * sizeof(float);  // red[][][][] in the kernel
  if (smem + static_smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(gemv_q4_tc_kernel<NP, KSL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return e;
  }
  const int ntiles = (R + 15) / 16;
  const int per_cta = 8 / KSL;
  const int blocks = std::max(1, std::min((ntiles + per_cta - 1) / per_cta, sms * 4));
  gemv_q4_tc_kernel<NP, KSL><<<blocks, 256, smem, st>>>(W, S, X, Y, R, K, M);
  return cudaGetLastError();
}

template <int NP>
static cudaError_t dispatch_tc(const uint8_t* W, const float* S, const float* X, float* Y, int R, int K, int M,
                               cudaStream_t st) {
  const int ntiles = (R + 15) / 16;
  // split the k groups of a tile over more warps when there are few tiles
  if (ntiles >= 4 * 148) return run_gemv_tc<NP, 1>(W, S, X, Y, R, K, M, st);
  if (ntiles >= 2 * 148) return run_gemv_tc<NP, 2>(W, S, X, Y, R, K, M, st);
  if (ntiles >= 148) return run_gemv_tc<NP, 4>(W, S, X, Y, R, K, M, st);
  return run_gemv_tc<NP, 8>(W, S, X, Y, R, K, M, st);
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

// Device word the streaming kernel raises when a bounded wait gives up (per device, never reset: a
// set flag means a copy did not complete, which does not happen on a healthy device).
static __device__ int g_gemv_err;
static int* gemv_err_flag() {
  void* p = nullptr;
  return cudaGetSymbolAddress(&p, g_gemv_err) == cudaSuccess ? (int*)p : nullptr;
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
  // Tensor-core path when its B-fragment table fits shared memory and the rows are 16-byte aligned.
  const int np = (n_act + 3) / 4;
  static const int use_tc = [] {
    const char* v = getenv("MLLM_GEMV_CUDA_CORES");
    return v && atoi(v) ? 0 : 1;
  }();
  if (use_tc && rows >= 2048 && !((uintptr_t)d_packed & 15) && !((uintptr_t)d_scales & 15) &&
      gemv_bulk_smem(cols, np) <= 200 * 1024) {
    int* err = gemv_err_flag();
    if (!err) return MLLM_ERR_CUDA;
    // one pass of tokens with a small K: two CTAs per SM with two stages each (2.6 % faster on the
    // 49152 x 576 lm_head shape than one CTA with three stages; the other shapes measured no better)
    if (np == 1 && gemv_bulk_smem(cols, 1, 2) <= kBulk2Smem)
      e = run_gemv_bulk<1, 2, 2, 2>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, err, st);
    else if (np == 1) e = run_gemv_bulk<1>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, err, st);
    else if (np == 2) e = run_gemv_bulk<2>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, err, st);
    else if (np == 3) e = run_gemv_bulk<3>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, err, st);
    else e = run_gemv_bulk<4>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, err, st);
    return e == cudaSuccess ? MLLM_OK : MLLM_ERR_CUDA;
  }
  if (use_tc && n_act > 1 && !((uintptr_t)d_packed & 15) && (size_t)np * (cols / 16) * 32 * 8 <= 192 * 1024) {
    if (np == 1) e = dispatch_tc<1>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, st);
    else if (np == 2) e = dispatch_tc<2>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, st);
    else if (np == 3) e = dispatch_tc<3>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, st);
    else e = dispatch_tc<4>(d_packed, d_scales, d_x, d_y, rows, cols, n_act, st);
    return e == cudaSuccess ? MLLM_OK : MLLM_ERR_CUDA;
  }
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
