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

// Four 8x8 fp16 matrices from shared memory: lane i gives the address of row i % 8 of matrix i / 8; lane
// (gid, t) receives elements (gid, 2t), (gid, 2t + 1) of each, i.e. for a token-major tile with the
// matrices at k offsets 0, 8, 16, 24 the B fragments of two k16 steps.
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* row) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(row);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
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

template <int TBW, int GPS>
struct GemmStage;
template <int TBW, int NS, int KS, class Rows, int GPS = 1, bool PDL = false>
__device__ __forceinline__ bool q4_gemm_core(const Rows& rows, const __half* __restrict__ Xhi,
                                             const __half* __restrict__ Xlo, int ldx, int K, int T, int t0,
                                             unsigned char* smem, float (&acc)[TBW][4],
                                             const int* skip = nullptr);

// Element-wise epilogue form: epi(tile_row, token, value) for every valid (row, token) of the tile.
template <int TBW, int NS = kStages, int KS = 1, class Rows, class Epi>
__device__ __forceinline__ void q4_gemm_rows(const Rows& rows, const __half* __restrict__ Xhi,
                                             const __half* __restrict__ Xlo, int ldx, int K, int T, int t0,
                                             unsigned char* smem, Epi epi) {
  float acc[TBW][4];
  q4_gemm_core<TBW, NS, KS, Rows, 1>(rows, Xhi, Xlo, ldx, K, T, t0, smem, acc);
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
// A pipeline stage carries GPS consecutive 32-wide k groups (one sync per stage).  KS > 1 splits the
// stages over KS groups of 4 warps (warp group w takes stages w, w + KS, ...), each with its own
// pipeline buffers and a named barrier; the partial sums are added, in group order, into group 0's
// accumulators (threads 0..127), which then hold the result.  Padded groups past the end load zero
// activations and scales, so they add nothing.
template <int TBW, int GPS>
struct GemmStage {
  static constexpr int BT = 8 * TBW;
  static constexpr int WROW = GPS * 16 + 16;       // bytes per weight row in smem (padded: conflict-free)
  static constexpr int XROW = GPS * 32 + 8;        // fp16 per token row in smem (padded)
  static constexpr size_t W = (size_t)kGemmRows * WROW;
  static constexpr size_t SC = (size_t)kGemmRows * GPS * 4;
  static constexpr size_t X = (size_t)BT * XROW * 2;  // bytes of one of hi / lo
  static constexpr size_t bytes = W + SC + 2 * X;
};

//
// PDL: the kernel was launched as a programmatic dependent of the previous kernel in the stream.  The
// weights and scales of the prologue stages (which no kernel writes) are requested first; then the
// CTA waits for the previous grid (griddepcontrol.wait) and, unless *skip is set, requests the
// activations.  Returns false, with every copy drained, when *skip is set.
template <int TBW, int NS, int KS, class Rows, int GPS, bool PDL>
__device__ __forceinline__ bool q4_gemm_core(const Rows& rows, const __half* __restrict__ Xhi,
                                             const __half* __restrict__ Xlo, int ldx, int K, int T, int t0,
                                             unsigned char* smem, float (&acc)[TBW][4], const int* skip) {
  using SG = GemmStage<TBW, GPS>;
  constexpr int kStages = NS;
  constexpr int BT = SG::BT;
  constexpr size_t kGroupBytes = (size_t)NS * SG::bytes;
  const int wg = KS > 1 ? (int)(threadIdx.x >> 7) : 0;
  const int lt = KS > 1 ? (int)(threadIdx.x & 127) : (int)threadIdx.x;
  const int lane = lt & 31, warp = lt >> 5;
  const int gid = lane >> 2, t = lane & 3;
  // k groups of this CTA: split blockIdx.z of gridDim.z (split-K across CTAs; 1 split normally)
  const int ngt = K >> 5;
  const int gbeg = (int)(((long)ngt * blockIdx.z) / gridDim.z), gend = (int)(((long)ngt * (blockIdx.z + 1)) / gridDim.z);
  const int nchunk = (gend - gbeg + GPS - 1) / GPS;                   // stages of GPS groups
  const int niter = nchunk > wg ? (nchunk - wg + KS - 1) / KS : 0;    // stages of this warp group
  unsigned char* base = smem + (size_t)wg * kGroupBytes;
  auto w_s = [&](int st) { return base + (size_t)st * SG::bytes; };
  auto s_s = [&](int st) { return reinterpret_cast<float*>(base + (size_t)st * SG::bytes + SG::W); };
  auto xh_s = [&](int st) { return reinterpret_cast<__half*>(base + (size_t)st * SG::bytes + SG::W + SG::SC); };
  auto xl_s = [&](int st) {
    return reinterpret_cast<__half*>(base + (size_t)st * SG::bytes + SG::W + SG::SC + SG::X);
  };
  auto sync = [&]() {
    if (KS == 1) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(1 + wg), "r"(kGemmThreads) : "memory");
  };
  // weights: 64 rows x GPS x 16 B; scales: 64 x GPS floats; activations: BT rows x GPS x 64 B x 2
  auto issue_w = [&](int i, int st) {
    const int g0 = gbeg + (wg + i * KS) * GPS;
    for (int j = lt; j < kGemmRows * GPS; j += kGemmThreads) {
      const int r = j / GPS, q = j % GPS, g = g0 + q;
      const bool ok = rows.valid(r) && g < gend;
      cp_async16(w_s(st) + r * SG::WROW + q * 16, rows.wrow(r) + min(g, gend - 1) * 16, ok);
      cp_async4(s_s(st) + r * GPS + q, rows.srow(r) + min(g, gend - 1), ok);
    }
  };
  auto issue_x = [&](int i, int st) {
    const int g0 = gbeg + (wg + i * KS) * GPS;
    for (int j = lt; j < BT * 4 * GPS; j += kGemmThreads) {  // 4 x 16 B per token row and group
      const int tk = j / (4 * GPS), c = j % (4 * GPS), g = g0 + (c >> 2);
      const int tok = t0 + tk;
      const bool ok = tok < T && g < gend;
      const size_t off = (size_t)min(tok, T - 1) * ldx + min(g, gend - 1) * 32 + (c & 3) * 8;
      cp_async16(xh_s(st) + tk * SG::XROW + c * 8, Xhi + off, ok);
      cp_async16(xl_s(st) + tk * SG::XROW + c * 8, Xlo + off, ok);
    }
  };
  auto issue = [&](int i, int st) {
    issue_w(i, st);
    issue_x(i, st);
  };
#pragma unroll
  for (int b = 0; b < TBW; ++b)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[b][i] = 0.f;
  // prologue (commit group s holds stage s's activations; group 0 also every prologue weight copy)
  if constexpr (PDL) {
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s)
      if (s < niter) issue_w(s, s);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (skip && *skip) {
      cp_async_commit();
      cp_async_wait<0>();
      return false;
    }
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < niter) issue_x(s, s);
      cp_async_commit();
    }
  } else {
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < niter) issue(s, s);
      cp_async_commit();
    }
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
#pragma unroll
    for (int q = 0; q < GPS; ++q) {
      const uint32_t* wr0 = reinterpret_cast<const uint32_t*>(w_s(st) + (warp * 16 + gid) * SG::WROW + q * 16);
      const uint32_t* wr1 = reinterpret_cast<const uint32_t*>(w_s(st) + (warp * 16 + gid + 8) * SG::WROW + q * 16);
      const float sc0 = s_s(st)[(warp * 16 + gid) * GPS + q];
      const float sc1 = s_s(st)[(warp * 16 + gid + 8) * GPS + q];
      uint32_t a0[4], a1[4];
      load_a_frag(wr0, wr1, 0, t, a0);
      load_a_frag(wr0, wr1, 1, t, a1);
#pragma unroll
      for (int b = 0; b < TBW; ++b) {
        // B fragments of both k16 steps, hi and lo: two ldmatrix.x4 (rows at lane % 8, k blocks at lane / 8)
        const int xo = (b * 8 + (lane & 7)) * SG::XROW + q * 32 + (lane >> 3) * 8;
        uint32_t bh[4], bl[4];
        ldsm_x4(bh, xh_s(st) + xo);
        ldsm_x4(bl, xl_s(st) + xo);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(d, a0, bh[0], bh[1]);
        mma16816(d, a0, bl[0], bl[1]);
        mma16816(d, a1, bh[2], bh[3]);
        mma16816(d, a1, bl[2], bl[3]);
        acc[b][0] = fmaf(sc0, d[0], acc[b][0]);
        acc[b][1] = fmaf(sc0, d[1], acc[b][1]);
        acc[b][2] = fmaf(sc1, d[2], acc[b][2]);
        acc[b][3] = fmaf(sc1, d[3], acc[b][3]);
      }
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
  return true;
}

template <int TBW, int NS = kStages, int KS = 1, int GPS = 1>
constexpr size_t q4_gemm_smem_bytes() {
  return (size_t)KS * NS * GemmStage<TBW, GPS>::bytes;
}

}  // namespace mllm
