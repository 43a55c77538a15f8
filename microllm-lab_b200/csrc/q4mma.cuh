// Tensor-core Q4 group-32 GEMM for token batches: Y[t][r] = sum_g sc[r][g] * sum_k (q[r][k]-8) * X[t][k]
// (engine/infer.js:88-116 applied to every token row).
//
// Weights stay in the PGW layout (packed rows [R][K/2] bytes, scales [R][K/32]); a CTA stages one
// 32-wide group of 64 rows (16 B per row) and 64 tokens per pipeline step in shared memory with
// cp.async, dequantises nibbles in registers straight into the A fragments of
// mma.sync.m16n8k16.f32.f16.f16.f32, and multiplies each group's partial sums by the fp32 scale.
//
// Exactness: (q - 8) is exact in fp16.  Activations are split x = hi + lo with hi = fp16(x),
// lo = fp16(x - hi) (relative residual <= 2^-22), both multiplied on the tensor cores and accumulated
// in fp32, so the result carries fp32-level error like the CUDA-core kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace mllm {

constexpr int kGemmRows = 64;     // weight rows per CTA (4 warps x 16)
constexpr int kGemmThreads = 128;
constexpr int kXPad = 40;         // fp16 per staged token row: 32 + 8 pad (conflict-free B loads)
constexpr int kStages = 3;         // default pipeline depth (32-wide k groups in flight)

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  const int n = pred ? 16 : 0;  // zero-fill when out of range
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool pred) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  const int n = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (lo nibble - 8, hi nibble - 8) of byte j of `w`, as an fp16 pair.  The byte lands in bytes 0 and
// 2; masking keeps lo (low half) and 16*hi (high half); 0x6400 makes 1024 + lo and 1024 + 16 hi;
// one fma scales the high half by 1/16 and removes the offsets.  Every step is exact in fp16.
__device__ __forceinline__ uint32_t nib_pair_f16(uint32_t w, int j) {
  const uint32_t v = __byte_perm(w, 0, (uint32_t)(j | (4 << 4) | (j << 8) | (4 << 12)));
  const uint32_t h = (v & 0x00F0000Fu) | 0x64006400u;
  const __half2 scale = __halves2half2(__float2half_rn(1.f), __float2half_rn(0.0625f));
  const __half2 off = __halves2half2(__float2half_rn(-1032.f), __float2half_rn(-72.f));
  const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), scale, off);
  return *reinterpret_cast<const uint32_t*>(&r);
}

// A fragment (16 rows x 16 k) for lane (gid, t) from the staged group: rows are 16-byte records
// (32 nibbles), k16 block `kb` is bytes 8kb..8kb+7 of a record.
__device__ __forceinline__ void load_a_frag(const uint32_t* wrow_gid, const uint32_t* wrow_gid8, int kb, int t,
                                            uint32_t (&a)[4]) {
  const uint2 r0 = *reinterpret_cast<const uint2*>(wrow_gid + 2 * kb);   // row gid: bytes 8kb..8kb+7
  const uint2 r1 = *reinterpret_cast<const uint2*>(wrow_gid8 + 2 * kb);  // row gid+8
  a[0] = nib_pair_f16(r0.x, t);  // row gid,   k 2t, 2t+1
  a[1] = nib_pair_f16(r1.x, t);  // row gid+8, k 2t, 2t+1
  a[2] = nib_pair_f16(r0.y, t);  // row gid,   k 2t+8, 2t+9
  a[3] = nib_pair_f16(r1.y, t);  // row gid+8, k 2t+8, 2t+9
}

// x -> (fp16 hi, fp16 lo) with hi + lo = x to ~2^-22 relative.
__device__ __forceinline__ void split_hi_lo(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// GEMM over a token batch.  X_hi/X_lo: fp16 [T][ldx] (k contiguous).  W: PGW packed rows, S: scales.
// Epilogue `epi(row, token, value)` is called for every (row < R, token < T) of the CTA's tile, from
// the lane that owns it.  TBW = 8-token blocks per warp (CTA covers 8 * TBW tokens).
// Row source of the default GEMM: tile row i -> matrix row r0 + i.
struct RowsLinear {
  const uint8_t* W;
  const float* S;
  int R, r0, half_k, ng;
  __device__ __forceinline__ bool valid(int i) const { return r0 + i < R; }
  __device__ __forceinline__ const uint8_t* wrow(int i) const { return W + (size_t)min(r0 + i, R - 1) * half_k; }
  __device__ __forceinline__ const float* srow(int i) const { return S + (size_t)min(r0 + i, R - 1) * ng; }
};

// Row source pairing two matrices with the same shape (w1 and w3): in each 16-row warp tile, rows
// 0..7 come from A and rows 8..15 from B at the same matrix rows, so the lane that owns row gid of A
// also owns row gid of B (accumulator elements 0/1 and 2/3).
struct RowsPaired {
  const uint8_t* WA;
  const float* SA;
  const uint8_t* WB;
  const float* SB;
  int R, r0, half_k, ng;  // r0: first matrix row of the CTA (32 per CTA)
  __device__ __forceinline__ int mrow(int i) const { return r0 + (i >> 4) * 8 + (i & 7); }
  __device__ __forceinline__ bool valid(int i) const { return mrow(i) < R; }
  __device__ __forceinline__ const uint8_t* wrow(int i) const {
    return ((i & 8) ? WB : WA) + (size_t)min(mrow(i), R - 1) * half_k;
  }
  __device__ __forceinline__ const float* srow(int i) const {
    return ((i & 8) ? SB : SA) + (size_t)min(mrow(i), R - 1) * ng;
  }
};

template <int TBW, int NS = kStages, int KS = 1, class Rows>
__device__ __forceinline__ void q4_gemm_core(const Rows& rows, const __half* __restrict__ Xhi,
                                             const __half* __restrict__ Xlo, int ldx, int K, int T, int t0,
                                             unsigned char* smem, float (&acc)[TBW][4]);

// Element-wise epilogue form: epi(tile_row, token, value) for every valid (row, token) of the tile.
template <int TBW, int NS = kStages, int KS = 1, class Rows, class Epi>
__device__ __forceinline__ void q4_gemm_rows(const Rows& rows, const __half* __restrict__ Xhi,
                                             const __half* __restrict__ Xlo, int ldx, int K, int T, int t0,
                                             unsigned char* smem, Epi epi) {
  float acc[TBW][4];
  q4_gemm_core<TBW, NS, KS>(rows, Xhi, Xlo, ldx, K, T, t0, smem, acc);
  if (KS > 1 && threadIdx.x >= kGemmThreads) return;  // the k-split partial sums are in group 0
  // lane (gid, t) owns tile rows gid, gid+8 of its warp and tokens 2t, 2t+1 of each 8-token block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int ia = warp * 16 + gid, ib = ia + 8;
  const bool va = rows.valid(ia), vb = rows.valid(ib);
#pragma unroll
  for (int b = 0; b < TBW; ++b) {
    const int ta = t0 + b * 8 + 2 * t, tb = ta + 1;
    if (va && ta < T) epi(ia, ta, acc[b][0]);
    if (va && tb < T) epi(ia, tb, acc[b][1]);
    if (vb && ta < T) epi(ib, ta, acc[b][2]);
    if (vb && tb < T) epi(ib, tb, acc[b][3]);
  }
}

template <int TBW, int NS = kStages, int KS = 1, class Epi>
__device__ __forceinline__ void q4_gemm_tile(const uint8_t* __restrict__ W, const float* __restrict__ S,
                                             const __half* __restrict__ Xhi, const __half* __restrict__ Xlo, int ldx,
                                             int R, int K, int T, int r0, int t0, unsigned char* smem, Epi epi) {
  const RowsLinear rows{W, S, R, r0, K >> 1, K >> 5};
  q4_gemm_rows<TBW, NS, KS>(rows, Xhi, Xlo, ldx, K, T, t0, smem, [&](int i, int t, float v) { epi(r0 + i, t, v); });
}

// Main loop: `rows` maps tile rows 0..63 to weight rows; acc[b][0..3] of lane (gid, t) hold tile rows
// (16 warp + gid, same, +8, +8) x tokens (t0 + 8b + 2t, +1, 2t, +1).  Ends with all copies drained.
// KS > 1 splits the k groups over KS groups of 4 warps (group w takes k groups w, w + KS, ...), each
// with its own pipeline buffers and a named barrier; the partial sums are added, in group order, into
// group 0's accumulators (threads 0..127), which then hold the result.
template <int TBW, int NS, int KS, class Rows>
__device__ __forceinline__ void q4_gemm_core(const Rows& rows, const __half* __restrict__ Xhi,
                                             const __half* __restrict__ Xlo, int ldx, int K, int T, int t0,
                                             unsigned char* smem, float (&acc)[TBW][4]) {
  constexpr int kStages = NS;
  constexpr int BT = 8 * TBW;  // tokens per CTA
  constexpr size_t kGroupBytes = (size_t)NS * kGemmRows * 16 + (size_t)NS * kGemmRows * 4 +
                                 2 * (size_t)NS * BT * kXPad * sizeof(__half);
  const int wg = KS > 1 ? (int)(threadIdx.x >> 7) : 0;
  const int lt = KS > 1 ? (int)(threadIdx.x & 127) : (int)threadIdx.x;
  const int lane = lt & 31, warp = lt >> 5;
  const int gid = lane >> 2, t = lane & 3;
  // k groups of this CTA: split blockIdx.z of gridDim.z (split-K across CTAs; 1 split normally)
  const int ngt = K >> 5;
  const int gbeg = (int)(((long)ngt * blockIdx.z) / gridDim.z), gend = (int)(((long)ngt * (blockIdx.z + 1)) / gridDim.z);
  const int ng = gend - gbeg;
  const int niter = ng > wg ? (ng - wg + KS - 1) / KS : 0;  // k groups of this warp group: wg, wg + KS, ...
  // stage layout (per warp group)
  uint8_t* w_s = smem + (size_t)wg * kGroupBytes;                        // [kStages][64][16]
  float* s_s = reinterpret_cast<float*>(w_s + kStages * kGemmRows * 16);  // [kStages][64]
  __half* xh_s = reinterpret_cast<__half*>(s_s + kStages * kGemmRows);    // [kStages][BT][kXPad]
  __half* xl_s = xh_s + kStages * BT * kXPad;
  auto sync = [&]() {
    if (KS == 1) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(1 + wg), "r"(kGemmThreads) : "memory");
  };
  auto issue = [&](int i, int st) {
    const int g = gbeg + wg + i * KS;
    // weights: 64 rows x 16 B, scales: 64 floats (16 x 16 B), activations: BT rows x 64 B x 2
    if (lt < kGemmRows) {
      cp_async16(w_s + (st * kGemmRows + lt) * 16, rows.wrow(lt) + g * 16, rows.valid(lt));
      // scales of a group are one float per row (stride ng)
      cp_async4(s_s + st * kGemmRows + lt, rows.srow(lt) + g, rows.valid(lt));
    }
    for (int j = lt; j < BT * 4; j += kGemmThreads) {  // 4 x 16 B per token row (32 fp16)
      const int tk = j >> 2, c = j & 3;
      const int tok = t0 + tk;
      const bool ok = tok < T;
      const size_t off = (size_t)min(tok, T - 1) * ldx + g * 32 + c * 8;
      cp_async16(xh_s + (st * BT + tk) * kXPad + c * 8, Xhi + off, ok);
      cp_async16(xl_s + (st * BT + tk) * kXPad + c * 8, Xlo + off, ok);
    }
  };
#pragma unroll
  for (int b = 0; b < TBW; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[b][i] = 0.f;
  // prologue
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < niter) issue(s, s);
    cp_async_commit();
  }
  for (int i = 0; i < niter; ++i) {
    cp_async_wait<kStages - 2>();
    sync();
    const int st = i % kStages;
    {
      const int in = i + kStages - 1;
      if (in < niter) issue(in, in % kStages);
      cp_async_commit();
    }
    const uint32_t* wr0 = reinterpret_cast<const uint32_t*>(w_s + (st * kGemmRows + warp * 16 + gid) * 16);
    const uint32_t* wr1 = reinterpret_cast<const uint32_t*>(w_s + (st * kGemmRows + warp * 16 + gid + 8) * 16);
    const float sc0 = s_s[st * kGemmRows + warp * 16 + gid];
    const float sc1 = s_s[st * kGemmRows + warp * 16 + gid + 8];
    uint32_t a0[4], a1[4];
    load_a_frag(wr0, wr1, 0, t, a0);
    load_a_frag(wr0, wr1, 1, t, a1);
#pragma unroll
    for (int b = 0; b < TBW; ++b) {
      const __half* xh = xh_s + (st * BT + b * 8 + gid) * kXPad + 2 * t;
      const __half* xl = xl_s + (st * BT + b * 8 + gid) * kXPad + 2 * t;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      mma16816(d, a0, *reinterpret_cast<const uint32_t*>(xh), *reinterpret_cast<const uint32_t*>(xh + 8));
      mma16816(d, a0, *reinterpret_cast<const uint32_t*>(xl), *reinterpret_cast<const uint32_t*>(xl + 8));
      mma16816(d, a1, *reinterpret_cast<const uint32_t*>(xh + 16), *reinterpret_cast<const uint32_t*>(xh + 24));
      mma16816(d, a1, *reinterpret_cast<const uint32_t*>(xl + 16), *reinterpret_cast<const uint32_t*>(xl + 24));
      acc[b][0] = fmaf(sc0, d[0], acc[b][0]);
      acc[b][1] = fmaf(sc0, d[1], acc[b][1]);
      acc[b][2] = fmaf(sc1, d[2], acc[b][2]);
      acc[b][3] = fmaf(sc1, d[3], acc[b][3]);
    }
  }
  cp_async_wait<0>();
  if (KS > 1) {
    __syncthreads();  // every group is done with its pipeline buffers
    float* red = reinterpret_cast<float*>(smem);  // [KS-1][128][TBW*4]
    if (wg > 0) {
#pragma unroll
      for (int b = 0; b < TBW; ++b)
#pragma unroll
        for (int i = 0; i < 4; ++i) red[((size_t)(wg - 1) * kGemmThreads + lt) * TBW * 4 + b * 4 + i] = acc[b][i];
    }
    __syncthreads();
    if (wg == 0) {
      for (int w = 1; w < KS; ++w)
#pragma unroll
        for (int b = 0; b < TBW; ++b)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[b][i] += red[((size_t)(w - 1) * kGemmThreads + lt) * TBW * 4 + b * 4 + i];
    }
  }
}

template <int TBW, int NS = kStages, int KS = 1>
constexpr size_t q4_gemm_smem_bytes() {
  return (size_t)KS * ((size_t)NS * kGemmRows * 16 + (size_t)NS * kGemmRows * 4 +
                       2 * (size_t)NS * (8 * TBW) * kXPad * sizeof(__half));
}

}  // namespace mllm
