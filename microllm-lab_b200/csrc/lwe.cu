// Layer-wise engine: forwards over a batch of T tokens that may belong to different sequence slots
// (each token has a slot, a position and an id).  Used for prefill (T prompt tokens of one slot,
// causal), the replicated multi-sequence decode (one token per slot per step) and batched verify.
//
// Per layer (engine/infer.js:553-577 applied to every token): norm1 + fp16 hi/lo split ->
// QKV GEMM -> RoPE + K/V cache write -> attention (one CTA per token and kv head, K/V rows read once
// for all heads of the group) -> proj GEMM + residual -> norm2 + split -> w1/w3 GEMM with SiLU*mul
// (GPT-2: fc + bias + GELU) -> w2 GEMM + residual.  Then norm_f + lm_head GEMM with an argmax
// epilogue (lowest index on ties, engine/infer.js:240-250) on the rows that need a next token.
// GEMMs run on the tensor cores (q4mma.cuh).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "device_common.cuh"
#include "engine.cuh"
#include "lwe.cuh"
#include "q4mma.cuh"
#include "tc5.cuh"

namespace mllm {

// Kernel launches issued by this thread (read by the runtime to report launches per call).
thread_local long g_lwe_launches = 0;
long lwe_launch_count() { return g_lwe_launches; }

// Programmatic dependent launch.  The forward's kernels are launched with programmatic stream
// serialisation: a kernel's CTAs start as soon as the previous grid's CTAs have exited, before that
// grid's memory flush, and wait for it with griddepcontrol.wait before they read or write any buffer
// that another kernel writes (the skip flag included).  The GEMMs request their first weight stages
// before that wait.  No kernel triggers its dependents early (an early trigger let the next grid's CTAs
// take SM slots during this grid's tail and unbalanced the GEMMs), and every kernel waits before it
// exits, so a grid's completion still implies its predecessors'.  Without the launch attribute the
// wait returns at once.
__device__ __forceinline__ void pdl_enter() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
thread_local bool g_lwe_pdl = true;
template <typename... P, typename... A>
static inline void lwe_launch(void (*k)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = g_lwe_pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
  ++g_lwe_launches;
}

// GEMM tiles: 64 weight rows x 8*TBW tokens per CTA; TBW is picked per launch so that small-R GEMMs
// still fill the GPU, and the k-pipeline is deeper for the smaller token tiles (all under 48 KB).
// The k groups may also be split over KS groups of 4 warps inside the CTA (more warps in flight per
// SM when a GEMM has few CTAs); the pipeline is deeper for the smaller tiles (all under 100 KB).
template <int TBW, int KSPLIT, bool LM = false>
struct LweTile {
  static constexpr int BT = 8 * TBW;
  static constexpr int KS = KSPLIT;
  // k groups per pipeline stage; the lm_head GEMM (thousands of CTAs) keeps small stages for occupancy
  static constexpr int GPS = LM ? 1 : (KS == 1 ? 4 : 2);
  static constexpr int NS = LM ? 4 : ((TBW == 8 && KS != 2) ? 2 : 3);
  static constexpr int THREADS = kGemmThreads * KS;
  static constexpr size_t smem() { return q4_gemm_smem_bytes<TBW, NS, KS, GPS>(); }
};

// 1 / RMS of token t from the per-row-tile partial sums of squares the previous GEMM left in a.ss
// (engine/infer.js:134-143 with the gain folded into the activations).
__device__ __forceinline__ float fold_inv(const LweArgs& a, int t) {
  const float* p = a.ss + (size_t)t * kLweSsStride;
  const int nt = (a.m.D + kGemmRows - 1) / kGemmRows;
  float s = 0.f;
  for (int j = 0; j < nt; ++j) s += p[j];
  return 1.f / sqrtf(s / a.m.D + 1e-6f);
}

// Split-K across CTAs (gridDim.z > 1, few-token GEMMs): each CTA leaves its partial tile in
// a.skws; the last CTA of a tile (counter a.skctr[tile], reset by it) adds the partials in split order
// and goes on to the epilogue, the others return false.  With gridDim.z == 1 it returns true at once.
template <int TBW>
__device__ __forceinline__ bool lwe_splitk(const LweArgs& a, float (&acc)[TBW][4]) {
  const int nz = gridDim.z;
  if (nz == 1) return true;
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  const bool g0 = threadIdx.x < kGemmThreads;
  float* mine = a.skws + (((size_t)tile * nz + blockIdx.z) * kGemmThreads + (threadIdx.x & (kGemmThreads - 1))) * TBW * 4;
  if (g0) {
#pragma unroll
    for (int b = 0; b < TBW; ++b) reinterpret_cast<float4*>(mine)[b] = make_float4(acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
  }
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int done = atomicAdd(&a.skctr[tile], 1) + 1;
    last = done == nz;
    if (last) a.skctr[tile] = 0;
  }
  __syncthreads();
  if (!last) return false;
  __threadfence();
  if (g0) {
#pragma unroll
    for (int b = 0; b < TBW; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
    for (int z = 0; z < nz; ++z) {
      const float* pz = a.skws + (((size_t)tile * nz + z) * kGemmThreads + threadIdx.x) * TBW * 4;
#pragma unroll
      for (int b = 0; b < TBW; ++b) {
        const float4 v = ldcg_f4(pz + 4 * b);
        acc[b][0] += v.x;
        acc[b][1] += v.y;
        acc[b][2] += v.z;
        acc[b][3] += v.w;
      }
    }
  }
  return true;
}

// Offset of activation element (t, k) in a GEMM-input buffer: row-major [T][ld], or the tiled layout of
// the tcgen05 tile (tc5::tiled_at) when the forward runs its GEMMs there (a.tiled).
__device__ __forceinline__ size_t act_off(const LweArgs& a, int T, int t, int k, int ld) {
  return a.tiled ? tc5::tiled_at(t, k, (T + 7) >> 3) : (size_t)t * ld + k;
}

// Element-wise epilogue over a 64-row tile (threads of the first warp group): epi(row, token, value).
template <int TBW, class Epi>
__device__ __forceinline__ void lwe_tile_epi(const float (&acc)[TBW][4], int r0, int t0, int R, int T, Epi epi) {
  if (threadIdx.x >= kGemmThreads) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int ra = r0 + warp * 16 + gid, rb = ra + 8;
#pragma unroll
  for (int b = 0; b < TBW; ++b) {
    const int ta = t0 + b * 8 + 2 * t, tb = ta + 1;
    if (ra < R && ta < T) epi(ra, ta, acc[b][0]);
    if (ra < R && tb < T) epi(ra, tb, acc[b][1]);
    if (rb < R && ta < T) epi(rb, ta, acc[b][2]);
    if (rb < R && tb < T) epi(rb, tb, acc[b][3]);
  }
}

// ---------------------------------------------------------------------------------------------
// RMSNorm (engine/infer.js:134-143) or LayerNorm (engine/infer.js:147-164) of one row by one warp,
// written as fp16 hi/lo.  The row (D <= 1024) is read once into registers through L2 (rows written by
// other CTAs of the same launch).
__device__ __forceinline__ void warp_norm_split(const float* x, int D, bool ln, const float* g, __half* oh,
                                                __half* ol) {
  const int lane = threadIdx.x & 31;
  float4 v[8];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = lane * 4 + i * 128;
    v[i] = k < D ? ldcg_f4(x + k) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s1 += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    s2 = fmaf(v[i].x, v[i].x, fmaf(v[i].y, v[i].y, fmaf(v[i].z, v[i].z, fmaf(v[i].w, v[i].w, s2))));
  }
  s1 = warp_sum(s1);
  float mean = 0.f, inv;
  if (!ln) {
    s2 = warp_sum(s2);
    inv = 1.f / sqrtf(s2 / D + 1e-6f);
  } else {
    mean = s1 / D;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = lane * 4 + i * 128;
      if (k < D) {
        var = fmaf(v[i].x - mean, v[i].x - mean, var);
        var = fmaf(v[i].y - mean, v[i].y - mean, var);
        var = fmaf(v[i].z - mean, v[i].z - mean, var);
        var = fmaf(v[i].w - mean, v[i].w - mean, var);
      }
    }
    var = warp_sum(var);
    inv = 1.f / sqrtf(var / D + 1e-5f);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = lane * 4 + i * 128;
    if (k >= D) break;
    const float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    const float4 gg = *reinterpret_cast<const float4*>(g + k);
    const float ga[4] = {gg.x, gg.y, gg.z, gg.w};
    __half hh[4], ll[4];
    if (!ln) {
#pragma unroll
      for (int j = 0; j < 4; ++j) split_hi_lo(e[j] * inv * ga[j], hh[j], ll[j]);
    } else {
      const float4 bb = *reinterpret_cast<const float4*>(g + D + k);
      const float ba[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) split_hi_lo(fmaf((e[j] - mean) * inv, ga[j], ba[j]), hh[j], ll[j]);
    }
    *reinterpret_cast<__half2*>(oh + k) = __halves2half2(hh[0], hh[1]);
    *reinterpret_cast<__half2*>(oh + k + 2) = __halves2half2(hh[2], hh[3]);
    *reinterpret_cast<__half2*>(ol + k) = __halves2half2(ll[0], ll[1]);
    *reinterpret_cast<__half2*>(ol + k + 2) = __halves2half2(ll[2], ll[3]);
  }
}

// Embedding of token t (one CTA per token); with g != nullptr also the first layer's norm1 into xh/xl.
__global__ void lwe_embed(const __grid_constant__ LweArgs a, int T, const float* g) {
  pdl_enter();
  if (a.skip && *a.skip) return;  // a finished speculative loop replays as no-ops
  const int t = blockIdx.x;
  if (t >= T) return;
  const ModelDev& md = a.m;
  const int D = md.D, pos = a.pos[t];
  int id = a.tok[t];
  if (id < 0 || id >= md.vocab) {  // device-resident prompts are checked here (error code 2)
    if (threadIdx.x == 0) atomicCAS(a.err, 0, 2);
    id = 0;
  }
  const uint8_t* row = reinterpret_cast<const uint8_t*>(md.lm.w) + (size_t)id * (D / 2);
  const float* sc = md.lm.s + (size_t)id * (D / 32);
  for (int k = threadIdx.x; k < D; k += blockDim.x) {
    const int b = row[k >> 1];
    float v = (float)(((k & 1) ? (b >> 4) : (b & 15)) - 8) * sc[k >> 5];  // engine/infer.js:395-415
    if (md.arch == 1) {                                                   // engine/infer.js:383-392, 416-419
      if (md.sf) v = __fdiv_rn(v, md.sf[k]);
      v += md.wpe[(size_t)min(pos, md.max_seq - 1) * D + k];
    }
    a.x[(size_t)t * D + k] = v;
  }
  if (g) {
    __syncthreads();
    if (threadIdx.x < 32) {
      const float* x = a.x + (size_t)t * D;
      __half* oh = a.xh + (size_t)t * a.ldx;
      __half* ol = a.xl + (size_t)t * a.ldx;
      if (a.fold) {  // x * gain as fp16 hi/lo, sum of squares for the consumer's 1/RMS
        float s2 = 0.f;
        for (int k = threadIdx.x; k < D; k += 32) {
          const float v = __ldcg(x + k);
          s2 = fmaf(v, v, s2);
          const size_t o = act_off(a, T, t, k, a.ldx);
          split_hi_lo(v * g[k], a.xh[o], a.xl[o]);
        }
        s2 = warp_sum(s2);
        const int nt = (D + kGemmRows - 1) / kGemmRows;
        if (threadIdx.x < nt) a.ss[(size_t)t * kLweSsStride + threadIdx.x] = threadIdx.x == 0 ? s2 : 0.f;
      } else {
        warp_norm_split(x, D, md.arch == 1, g, oh, ol);
      }
    }
  }
}

// RMSNorm / LayerNorm of X[src[i]] (or X[i]) -> fp16 hi/lo rows i of xh/xl.  One CTA per row.  TILED
// writes xh3/xl3 instead, in the 8-token-block layout the tcgen05 tile reads (tc5::tiled_at).
template <bool TILED>
__global__ void lwe_norm_split(const __grid_constant__ LweArgs a, int T, const float* g, const int* src) {
  pdl_enter();
  if (a.skip && *a.skip) return;  // a finished speculative loop replays as no-ops
  const int i = blockIdx.x;
  if (i >= T) return;
  const ModelDev& md = a.m;
  const int D = md.D;
  const int row = src ? src[i] : i;
  const float* x = a.x + (size_t)row * D;
  __shared__ float red[2][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  float s1 = 0.f, s2 = 0.f;
  for (int k = threadIdx.x; k < D; k += blockDim.x) {
    s1 += x[k];
    s2 = fmaf(x[k], x[k], s2);
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) {
    red[0][warp] = s1;
    red[1][warp] = s2;
  }
  __syncthreads();
  s1 = 0.f;
  s2 = 0.f;
  for (int w = 0; w < nw; ++w) {
    s1 += red[0][w];
    s2 += red[1][w];
  }
  __half* oh = TILED ? a.xh3 : a.xh + (size_t)i * a.ldx;
  __half* ol = TILED ? a.xl3 : a.xl + (size_t)i * a.ldx;
  const int T8 = (T + 7) / 8;
  auto at = [&](int k) -> size_t { return TILED ? tc5::tiled_at(i, k, T8) : (size_t)k; };
  if (md.arch == 0) {
    const float inv = 1.f / sqrtf(s2 / D + 1e-6f);  // engine/infer.js:134-143
    for (int k = threadIdx.x; k < D; k += blockDim.x) split_hi_lo(x[k] * inv * g[k], oh[at(k)], ol[at(k)]);
  } else {
    const float mean = s1 / D;  // engine/infer.js:147-164 (second pass for the variance)
    float v = 0.f;
    for (int k = threadIdx.x; k < D; k += blockDim.x) {
      const float d = x[k] - mean;
      v = fmaf(d, d, v);
    }
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[0][warp] = v;
    __syncthreads();
    v = 0.f;
    for (int w = 0; w < nw; ++w) v += red[0][w];
    const float inv = 1.f / sqrtf(v / D + 1e-5f);
    for (int k = threadIdx.x; k < D; k += blockDim.x)
      split_hi_lo(fmaf((x[k] - mean) * inv, g[k], g[D + k]), oh[at(k)], ol[at(k)]);
  }
}

// QKV GEMM: qkv[t][r] = W_qkv[r] . norm1(x_t) (+ bias).  With a.fold the activations are x * gain and
// the token's 1/RMS multiplies the result.  With rope != 0 the epilogue also does what lwe_rope_kv does
// (RoPE on the q and k heads at each token's position, K/V cache rows written): a 64-row tile is one
// head of the [q heads | k heads | v heads] layout, staged in shared memory so that both halves of each
// rotated pair are at hand.
template <int TBW, int KS>
__global__ void __launch_bounds__(LweTile<TBW, KS>::THREADS) lwe_gemm_qkv(const __grid_constant__ LweArgs a, int T,
                                                                         int l, int rope) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LweTile<TBW, KS>;
  __shared__ float sinv[C::BT];
  const LayerDev& L = a.m.layers[l];
  const int R = a.m.QKV, K = a.m.D, t0 = blockIdx.y * C::BT;
  const float* bias = L.qkv_b;
  float* out = a.qkv;
  const int r0 = blockIdx.x * kGemmRows;
  const RowsLinear rows{reinterpret_cast<const uint8_t*>(L.qkv.w), L.qkv.s, R, r0, K >> 1, K >> 5};
  float acc[TBW][4];
  // waits for the previous kernel inside, after requesting the first weight stages
  if (!q4_gemm_core<TBW, C::NS, C::KS, decltype(rows), C::GPS, true>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc,
                                                                     a.skip))
    return;  // a finished speculative loop replays as no-ops
  if (!lwe_splitk<TBW>(a, acc)) return;
  if (threadIdx.x < C::BT) sinv[threadIdx.x] = a.fold && t0 + (int)threadIdx.x < T ? fold_inv(a, t0 + threadIdx.x) : 1.f;
  __syncthreads();  // also: every warp is done with the pipeline buffers
  if (!rope) {
    lwe_tile_epi<TBW>(acc, r0, t0, R, T, [&](int r, int t, float v) {
      v *= sinv[t - t0];
      out[(size_t)t * R + r] = bias ? v + bias[r] : v;
    });
    return;
  }
  constexpr int TS = C::BT + 1;  // padded: conflict-free column reads
  float* tile = reinterpret_cast<float*>(smem);  // [64][TS]
  lwe_tile_epi<TBW>(acc, r0, t0, R, T, [&](int r, int t, float v) {
    v *= sinv[t - t0];
    tile[(r - r0) * TS + (t - t0)] = bias ? v + bias[r] : v;
  });
  __syncthreads();
  const ModelDev& md = a.m;
  const int D = md.D, NKV = md.NKV;
  const int kind = r0 < D ? 0 : (r0 < D + NKV * 64 ? 1 : 2);  // q, k or v head
  const int g = kind == 1 ? (r0 - D) >> 6 : (kind == 2 ? (r0 - D - NKV * 64) >> 6 : 0);
  const int half = kind < 2 && md.arch == 0 ? md.rope_dim / 2 : 0;
  for (int i = threadIdx.x; i < 64 * C::BT; i += blockDim.x) {
    const int tl = i >> 6, d = i & 63, t = t0 + tl;
    if (t >= T) continue;
    float v = tile[d * TS + tl];
    const int pos = a.pos[t];
    if (d < 2 * half) {  // engine/infer.js:436-456, the operation order of lwe_rope_kv
      const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
      const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
      if (d < half)
        v = fmaf(-tile[(d + half) * TS + tl], sn[d], v * cs[d]);
      else
        v = fmaf(tile[(d - half) * TS + tl], sn[d], v * cs[d]);
    }
    out[(size_t)t * R + r0 + d] = v;
    if (kind > 0)  // engine/infer.js:457-464
      (kind == 1 ? a.kc : a.vc)[a.slot[t]][(((size_t)l * NKV + g) * md.kv_len + pos) * 64 + d] = v;
  }
}

// RoPE on k (and on the q heads of the group) at each token's position, then the K/V cache write
// (engine/infer.js:436-464).  grid (T, NKV), 64 threads: thread d < 32 rotates pair (d, d + 32).
__global__ void lwe_rope_kv(const __grid_constant__ LweArgs a, int T) {
  pdl_enter();
  if (a.skip && *a.skip) return;  // a finished speculative loop replays as no-ops
  const int t = blockIdx.x, g = blockIdx.y;
  if (t >= T) return;
  const ModelDev& md = a.m;
  const int D = md.D, NKV = md.NKV, rep = md.NH / NKV, pos = a.pos[t];
  float* row = a.qkv + (size_t)t * md.QKV;
  float* k = row + D + g * 64;
  const float* v = row + D + NKV * 64 + g * 64;
  const int d = threadIdx.x;
  if (md.arch == 0 && md.rope_dim > 0) {
    const int half = md.rope_dim / 2;
    if (d < half) {
      const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
      const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
      for (int h = -1; h < rep; ++h) {  // h = -1: the key, else query head g * rep + h
        float* p = h < 0 ? k : row + (g * rep + h) * 64;
        const float a0 = p[d], a1 = p[d + half];
        p[d] = fmaf(-a1, sn[d], a0 * cs[d]);
        p[d + half] = fmaf(a0, sn[d + half], a1 * cs[d + half]);
      }
    }
    __syncthreads();
  }
  const int slot = a.slot[t];
  const size_t kv = (((size_t)a.layer * NKV + g) * md.kv_len + pos) * 64;
  a.kc[slot][kv + d] = k[d];
  a.vc[slot][kv + d] = v[d];
}

// Attention of the REP query heads of kv head g for token t over positions 0..pos[t] of its slot
// (engine/infer.js:466-495).  grid (T, NKV), 128 threads.  Three passes over shared memory:
// scores (one thread per position, the K row read as 16 float4, q broadcast from shared memory),
// softmax per head (one warp per head), then P.V (16 threads per row of V, 8 position lanes, 8 rows
// in flight per thread).  Output rows are written as fp16 hi/lo into xh/xl for the proj GEMM.
// FUSED (every token of the launch in its own slot, as in a batched decode step): the CTA also applies
// RoPE to its q heads and k (engine/infer.js:436-458) and writes the token's K/V row into the cache
// (engine/infer.js:459-464) before reading the cache; otherwise lwe_rope_kv ran first.
constexpr int kAttnThreads = 128;
constexpr int kAttnLanes = kAttnThreads / 16;  // position lanes of the P.V pass
template <int REP, bool FUSED>
__global__ void __launch_bounds__(kAttnThreads) lwe_attention(const __grid_constant__ LweArgs a, int T) {
  pdl_enter();
  if (a.skip && *a.skip) return;  // a finished speculative loop replays as no-ops
  extern __shared__ __align__(16) float asm_[];
  const int t = blockIdx.x, g = blockIdx.y;
  if (t >= T) return;
  const ModelDev& md = a.m;
  const int NKV = md.NKV, pos = a.pos[t], npos = pos + 1, kvs = md.kv_len;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* qs = asm_;                  // [REP][64]
  float* sc = qs + REP * 64;         // [REP][kv_len]
  float* red = sc + ((REP * kvs + 3) & ~3);  // [kAttnLanes][REP][64], 16-byte aligned (float4 stores)
  __shared__ float inv_sum[REP];
  __shared__ float ks[64];
  const float* qrow = a.qkv + (size_t)t * md.QKV + g * REP * 64;
  const size_t base = ((size_t)a.layer * NKV + g) * md.kv_len * 64;
  float* kcw = a.kc[a.slot[t]] + base;
  float* vcw = a.vc[a.slot[t]] + base;
  for (int i = tid; i < REP * 64; i += kAttnThreads) qs[i] = qrow[i];
  if (FUSED) {
    const float* krow = a.qkv + (size_t)t * md.QKV + md.D + g * 64;
    const float* vrow = krow + NKV * 64;
    if (tid < 64) {
      ks[tid] = krow[tid];
      vcw[(size_t)pos * 64 + tid] = vrow[tid];
    }
    __syncthreads();
    if (md.arch == 0 && md.rope_dim > 0) {
      const int half = md.rope_dim / 2;
      const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
      const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
      // thread (h, d): h = -1 is the key, else query head h of the group; pair (d, d + half)
      for (int i = tid; i < (REP + 1) * half; i += kAttnThreads) {
        const int h = i / half - 1, d = i % half;
        float* p = h < 0 ? ks : qs + h * 64;
        const float a0 = p[d], a1 = p[d + half];
        p[d] = fmaf(-a1, sn[d], a0 * cs[d]);
        p[d + half] = fmaf(a0, sn[d + half], a1 * cs[d + half]);
      }
      __syncthreads();
    }
    if (tid < 64) kcw[(size_t)pos * 64 + tid] = ks[tid];
  }
  const float* kc = kcw;
  const float* vc = vcw;
  __syncthreads();
  // scores (engine/infer.js:470-476: f32(dot * 1/sqrt(64)))
  for (int p = tid; p < npos; p += kAttnThreads) {
    const float4* kr = reinterpret_cast<const float4*>(kc + (size_t)p * 64);
    float4 kk[16];
    // L1-cached loads: a warp's 16 loads walk 32 rows, so each 32-byte sector serves two of them
    // (the only row this kernel writes, at pos, is read after the __syncthreads above)
#pragma unroll
    for (int j = 0; j < 16; ++j) kk[j] = kr[j];
    float s[REP];
#pragma unroll
    for (int h = 0; h < REP; ++h) {
      s[h] = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float4 q = reinterpret_cast<const float4*>(qs + h * 64)[j];
        s[h] = fmaf(q.x, kk[j].x, s[h]);
        s[h] = fmaf(q.y, kk[j].y, s[h]);
        s[h] = fmaf(q.z, kk[j].z, s[h]);
        s[h] = fmaf(q.w, kk[j].w, s[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < REP; ++h) sc[h * kvs + p] = s[h] * 0.125f;
  }
  __syncthreads();
  // softmax per head (engine/infer.js:477-486)
  if (warp < REP) {
    float* row = sc + warp * kvs;
    float m = -INFINITY;
    for (int p = lane; p < npos; p += 32) m = fmaxf(m, row[p]);
    m = warp_max(m);
    float sum = 0.f;
    for (int p = lane; p < npos; p += 32) {
      const float e = expf(row[p] - m);
      row[p] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) inv_sum[warp] = 1.f / sum;
  }
  __syncthreads();
  // P.V (engine/infer.js:487-495): thread = (position lane pl, float4 column dq)
  {
    const int pl = tid >> 4, dq = tid & 15;
    float4 acc[REP];
#pragma unroll
    for (int h = 0; h < REP; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int kVU = 8;  // V rows in flight per thread (16 measured 8 % slower)
    for (int p0 = pl; p0 < npos; p0 += kVU * kAttnLanes) {
      float4 vv[kVU];
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int p = min(p0 + kAttnLanes * u, pos);
        vv[u] = ldcg_f4(vc + (size_t)p * 64 + dq * 4);
      }
#pragma unroll
      for (int u = 0; u < kVU; ++u) {
        const int p = p0 + kAttnLanes * u;
        if (p < npos) {
#pragma unroll
          for (int h = 0; h < REP; ++h) {
            const float e = sc[h * kvs + p];
            acc[h].x = fmaf(e, vv[u].x, acc[h].x);
            acc[h].y = fmaf(e, vv[u].y, acc[h].y);
            acc[h].z = fmaf(e, vv[u].z, acc[h].z);
            acc[h].w = fmaf(e, vv[u].w, acc[h].w);
          }
        }
      }
    }
#pragma unroll
    for (int h = 0; h < REP; ++h) reinterpret_cast<float4*>(red + (pl * REP + h) * 64)[dq] = acc[h];
  }
  __syncthreads();
  for (int hd = tid; hd < REP * 64; hd += kAttnThreads) {
    const int h = hd >> 6, d = hd & 63;
    float r = 0.f;
#pragma unroll
    for (int q = 0; q < kAttnLanes; ++q) r += red[(q * REP + h) * 64 + d];
    const size_t off = act_off(a, T, t, (g * REP + h) * 64 + d, a.ldx);
    split_hi_lo(r * inv_sum[h], a.xh[off], a.xl[off]);
  }
}

// Decode-step attention split over positions (flash-decoding): grid (T, NKV, S), 64 threads; split sp
// covers positions [sp*64, sp*64 + 64) of 0..pos[t].  The split's K and V rows (contiguous in the
// cache) come into shared memory with two bulk copies while the CTA loads and rotates q.  Every token
// is in its own slot: the split holding position pos applies RoPE to k (engine/infer.js:436-458),
// writes the K/V row to the cache (engine/infer.js:459-464) and patches it into its staged copy.
// Each split leaves (max, sum, P.V) per head in `part`; the last split to finish (counter
// ctr[t*NKV+g], reset by it) merges them in split order and writes the heads' outputs as fp16 hi/lo
// into xh/xl.
constexpr int kAttnChunk = 64;
template <int REP, bool FUSED>
__global__ void __launch_bounds__(64) lwe_attn_split(const __grid_constant__ LweArgs a, int T, float* part, int* ctr) {
  pdl_enter();
  if (a.skip && *a.skip) return;  // a finished speculative loop replays as no-ops
  extern __shared__ __align__(128) float kvs[];  // K [64][64], V [64][64]
  const int t = blockIdx.x, g = blockIdx.y, sp = blockIdx.z, S = gridDim.z;
  const ModelDev& md = a.m;
  const int NKV = md.NKV, pos = a.pos[t], npos = pos + 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int p0 = sp * kAttnChunk, p1 = min(npos, p0 + kAttnChunk), n = p1 - p0;
  float* kb = kvs;
  float* vb = kvs + kAttnChunk * 64;
  __shared__ __align__(16) float qs[REP * 64];
  __shared__ float ks[64];
  __shared__ float sc[REP][kAttnChunk];
  __shared__ __align__(16) float red[4][REP][64];
  __shared__ float mx[REP], ls[REP];
  __shared__ int last;
  __shared__ __align__(8) uint64_t bar;
  const size_t base = ((size_t)a.layer * NKV + g) * md.kv_len * 64;
  float* kcw = a.kc[a.slot[t]] + base;
  float* vcw = a.vc[a.slot[t]] + base;
  float* mypart = part + (((size_t)t * NKV + g) * S + sp) * REP * 66;
  if (n > 0) {
    const bool owner = FUSED && p1 == npos;
    if (tid == 0) {
      mbar_init(&bar, 1);
      mbar_init_fence();
    }
    __syncthreads();
    if (tid == 0) {
      mbar_expect_tx(&bar, 2u * n * 256u);
      bulk_g2s(kb, kcw + (size_t)p0 * 64, n * 256u, &bar);
      bulk_g2s(vb, vcw + (size_t)p0 * 64, n * 256u, &bar);
    }
    const float* qrow = a.qkv + (size_t)t * md.QKV + g * REP * 64;
    for (int i = tid; i < REP * 64; i += 64) qs[i] = qrow[i];
    float vnew = 0.f;
    if (owner) {
      const float* krow = a.qkv + (size_t)t * md.QKV + md.D + g * 64;
      ks[tid] = krow[tid];
      vnew = krow[NKV * 64 + tid];
      vcw[(size_t)pos * 64 + tid] = vnew;
    }
    __syncthreads();
    if (FUSED && md.arch == 0 && md.rope_dim > 0) {  // unfused: lwe_rope_kv rotated q and wrote K/V
      const int half = md.rope_dim / 2;
      const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
      const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
      for (int i = tid; i < (REP + 1) * half; i += 64) {
        const int h = i / half - 1, d = i % half;
        if (h < 0 && !owner) continue;
        float* q = h < 0 ? ks : qs + h * 64;
        const float a0 = q[d], a1 = q[d + half];
        q[d] = fmaf(-a1, sn[d], a0 * cs[d]);
        q[d + half] = fmaf(a0, sn[d + half], a1 * cs[d + half]);
      }
      __syncthreads();
    }
    if (owner) kcw[(size_t)pos * 64 + tid] = ks[tid];
    if (!mbar_wait_bounded(&bar, 0, kWaitNs)) {
      atomicCAS(a.err, 0, 1);
      mbar_wait_bounded(&bar, 0, kWaitNs);  // the copies must land before the CTA may leave
    }
    if (owner) {  // the staged row at pos is the one written above
      kb[(pos - p0) * 64 + tid] = ks[tid];
      vb[(pos - p0) * 64 + tid] = vnew;
    }
    __syncthreads();
    // scores (engine/infer.js:470-476): thread = position; float4 chunks visited in a rotated order
    // so that the 8 threads of a shared-memory wavefront hit different banks
    if (tid < n) {
      const float4* kr = reinterpret_cast<const float4*>(kb + tid * 64);
      float acc[REP];
#pragma unroll
      for (int h = 0; h < REP; ++h) acc[h] = 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int c = (j + tid) & 15;
        const float4 k4 = kr[c];
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          const float4 q = reinterpret_cast<const float4*>(qs + h * 64)[c];
          acc[h] = fmaf(q.x, k4.x, acc[h]);
          acc[h] = fmaf(q.y, k4.y, acc[h]);
          acc[h] = fmaf(q.z, k4.z, acc[h]);
          acc[h] = fmaf(q.w, k4.w, acc[h]);
        }
      }
#pragma unroll
      for (int h = 0; h < REP; ++h) sc[h][tid] = acc[h] * 0.125f;
    }
    __syncthreads();
    // partial softmax per head
    for (int h = warp; h < REP; h += 2) {
      float m = -INFINITY;
      for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[h][i]);
      m = warp_max(m);
      float sum = 0.f;
      for (int i = lane; i < n; i += 32) {
        const float e = expf(sc[h][i] - m);
        sc[h][i] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        mx[h] = m;
        ls[h] = sum;
      }
    }
    __syncthreads();
    // P.V over the split: thread = (position lane pl of 4, float4 column dq)
    {
      const int pl = tid >> 4, dq = tid & 15;
      float4 acc[REP];
#pragma unroll
      for (int h = 0; h < REP; ++h) acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int i = pl; i < n; i += 4) {
        const float4 v = reinterpret_cast<const float4*>(vb + i * 64)[dq];
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          const float e = sc[h][i];
          acc[h].x = fmaf(e, v.x, acc[h].x);
          acc[h].y = fmaf(e, v.y, acc[h].y);
          acc[h].z = fmaf(e, v.z, acc[h].z);
          acc[h].w = fmaf(e, v.w, acc[h].w);
        }
      }
#pragma unroll
      for (int h = 0; h < REP; ++h) reinterpret_cast<float4*>(red[pl][h])[dq] = acc[h];
    }
    __syncthreads();
    for (int hd = tid; hd < REP * 64; hd += 64) {
      const int h = hd >> 6, d = hd & 63;
      mypart[h * 66 + 2 + d] = (red[0][h][d] + red[1][h][d]) + (red[2][h][d] + red[3][h][d]);
    }
    if (tid < REP) {
      mypart[tid * 66] = mx[tid];
      mypart[tid * 66 + 1] = ls[tid];
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int c = t * NKV + g;
    const int done = atomicAdd(&ctr[c], 1) + 1;
    last = done == S;
    if (last) ctr[c] = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge (engine/infer.js:477-495 over the whole range), splits in order
  const int nsp = (npos + kAttnChunk - 1) / kAttnChunk;
  const float* tp = part + ((size_t)t * NKV + g) * S * REP * 66;
  for (int hd = tid; hd < REP * 64; hd += 64) {
    const int h = hd >> 6, d = hd & 63;
    float M = -INFINITY;
    for (int q = 0; q < nsp; ++q) M = fmaxf(M, __ldcg(tp + (q * REP + h) * 66));
    float L = 0.f, O = 0.f;
    for (int q = 0; q < nsp; ++q) {
      const float* pq = tp + (q * REP + h) * 66;
      const float f = expf(__ldcg(pq) - M);
      L = fmaf(__ldcg(pq + 1), f, L);
      O = fmaf(__ldcg(pq + 2 + d), f, O);
    }
    const size_t off = act_off(a, T, t, (g * REP + h) * 64 + d, a.ldx);
    split_hi_lo(O / L, a.xh[off], a.xl[off]);
  }
}

// Positions per split of the decode attention and the split count for a cache of kv_len positions.
void lwe_attn_split_shape(int kv_len, int* chunk, int* splits) {
  *chunk = kAttnChunk;
  *splits = (kv_len + kAttnChunk - 1) / kAttnChunk;
}

static size_t attention_smem(int rep, int kv_len) {
  return (size_t)(rep * 64 + ((rep * kv_len + 3) & ~3) + kAttnLanes * rep * 64) * 4;
}

// GEMM with a residual epilogue: x[t][r] += W[r] . in_t (+ bias)  (proj and w2).  With gn != nullptr
// (folded RMSNorm) the epilogue also writes (x * gn) as fp16 hi/lo into nh/nl (stride ldn) and this
// row tile's sum of squares of the new x per token into a.ss[t][blockIdx.x].
template <int TBW, int KS>
__global__ void __launch_bounds__(LweTile<TBW, KS>::THREADS) lwe_gemm_resid(const __grid_constant__ LweArgs a, int T,
                                                                           Q4 w, const float* bias, int K,
                                                                           const float* gn, __half* nh, __half* nl,
                                                                           int ldn) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LweTile<TBW, KS>;
  __shared__ float ssw[4][C::BT];
  const int R = a.m.D, r0 = blockIdx.x * kGemmRows, t0 = blockIdx.y * C::BT;
  float* x = a.x;
  const RowsLinear rows{reinterpret_cast<const uint8_t*>(w.w), w.s, R, r0, K >> 1, K >> 5};
  float acc[TBW][4];
  // waits for the previous kernel inside, after requesting the first weight stages
  if (!q4_gemm_core<TBW, C::NS, C::KS, decltype(rows), C::GPS, true>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc,
                                                                     a.skip))
    return;  // a finished speculative loop replays as no-ops
  if (!lwe_splitk<TBW>(a, acc)) return;
  if (threadIdx.x < kGemmThreads) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, tq = lane & 3;
    const int ra = r0 + warp * 16 + gid, rb = ra + 8;
    const bool va = ra < R, vb = rb < R;
#pragma unroll
    for (int b = 0; b < TBW; ++b) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int tl = b * 8 + 2 * tq + e, tok = t0 + tl;
        float sq = 0.f;
        if (tok < T) {
          if (va) {
            float* px = x + (size_t)tok * R + ra;
            const float xn = *px + (bias ? acc[b][e] + bias[ra] : acc[b][e]);
            *px = xn;
            if (gn) {
              split_hi_lo(xn * gn[ra], nh[(size_t)tok * ldn + ra], nl[(size_t)tok * ldn + ra]);
              sq = xn * xn;
            }
          }
          if (vb) {
            float* px = x + (size_t)tok * R + rb;
            const float xn = *px + (bias ? acc[b][2 + e] + bias[rb] : acc[b][2 + e]);
            *px = xn;
            if (gn) {
              split_hi_lo(xn * gn[rb], nh[(size_t)tok * ldn + rb], nl[(size_t)tok * ldn + rb]);
              sq = fmaf(xn, xn, sq);
            }
          }
        }
        if (gn) {
          sq += __shfl_xor_sync(0xffffffffu, sq, 4);
          sq += __shfl_xor_sync(0xffffffffu, sq, 8);
          sq += __shfl_xor_sync(0xffffffffu, sq, 16);
          if (gid == 0) ssw[warp][tl] = sq;
        }
      }
    }
  }
  if (gn) {
    __syncthreads();
    if (threadIdx.x < C::BT && t0 + (int)threadIdx.x < T) {
      const int i = threadIdx.x;
      a.ss[(size_t)(t0 + i) * kLweSsStride + blockIdx.x] = (ssw[0][i] + ssw[1][i]) + (ssw[2][i] + ssw[3][i]);
    }
  }
}

// w1/w3 paired GEMM with the SiLU*mul epilogue (engine/infer.js:178-183, 522-524); output written as
// fp16 hi/lo into the second activation buffer (xh2/xl2).  32 matrix rows per CTA.
template <int TBW, int KS>
__global__ void __launch_bounds__(LweTile<TBW, KS>::THREADS) lwe_gemm_w13(const __grid_constant__ LweArgs a, int T,
                                                                         int l) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LweTile<TBW, KS>;
  __shared__ float sinv[C::BT];
  const LayerDev& L = a.m.layers[l];
  const int FF = a.m.FF, K = a.m.D;
  const RowsPaired rows{reinterpret_cast<const uint8_t*>(L.w1.w), L.w1.s, reinterpret_cast<const uint8_t*>(L.w3.w),
                        L.w3.s, FF, (int)blockIdx.x * 32, K >> 1, K >> 5};
  float acc[TBW][4];
  const int t0 = blockIdx.y * C::BT;
  // waits for the previous kernel inside, after requesting the first weight stages
  if (!q4_gemm_core<TBW, C::NS, C::KS, decltype(rows), C::GPS, true>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc,
                                                                     a.skip))
    return;  // a finished speculative loop replays as no-ops
  if (!lwe_splitk<TBW>(a, acc)) return;
  {
    const int tt = t0 + threadIdx.x;
    if (threadIdx.x < C::BT) sinv[threadIdx.x] = a.fold && tt < T ? fold_inv(a, tt) : 1.f;
    __syncthreads();
  }
  if (threadIdx.x >= kGemmThreads) return;  // partial sums were added into the first warp group
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int ia = warp * 16 + gid;  // A row (w1); the B row (w3) of the same matrix row is ia + 8
  if (!rows.valid(ia)) return;
  const int r = rows.mrow(ia);
#pragma unroll
  for (int b = 0; b < TBW; ++b) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tok = t0 + b * 8 + 2 * t + e;
      if (tok >= T) continue;
      const float iv = sinv[b * 8 + 2 * t + e];
      const float u = acc[b][e] * iv, v = acc[b][2 + e] * iv;
      const size_t off = (size_t)tok * a.ldx2 + r;
      split_hi_lo((u / (1.f + expf(-u))) * v, a.xh2[off], a.xl2[off]);
    }
  }
}

// GPT-2 fc GEMM with bias + GELU (engine/infer.js:512-515, 166-171) -> fp16 hi/lo (xh2/xl2)
template <int TBW, int KS>
__global__ void __launch_bounds__(LweTile<TBW, KS>::THREADS) lwe_gemm_fc(const __grid_constant__ LweArgs a, int T,
                                                                        int l) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LweTile<TBW, KS>;
  const LayerDev& L = a.m.layers[l];
  const int FF = a.m.FF, K = a.m.D;
  const float* bias = L.fc_b;
  const int r0 = blockIdx.x * kGemmRows, t0 = blockIdx.y * C::BT;
  const RowsLinear rows{reinterpret_cast<const uint8_t*>(L.w1.w), L.w1.s, FF, r0, K >> 1, K >> 5};
  float acc[TBW][4];
  // waits for the previous kernel inside, after requesting the first weight stages
  if (!q4_gemm_core<TBW, C::NS, C::KS, decltype(rows), C::GPS, true>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc,
                                                                     a.skip))
    return;  // a finished speculative loop replays as no-ops
  if (!lwe_splitk<TBW>(a, acc)) return;
  lwe_tile_epi<TBW>(acc, r0, t0, FF, T, [&](int r, int t, float v) {
    if (bias) v += bias[r];
    const float gl = 0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
    split_hi_lo(gl, a.xh2[(size_t)t * a.ldx2 + r], a.xl2[(size_t)t * a.ldx2 + r]);
  });
}

// Wide lm_head GEMM for many rows (a batched decode step) without a logits output.  One CTA per SM:
// the CTA's 8*TBW token rows of xh/xl stay in shared memory for the whole launch while its run of
// 64-row vocab tiles streams through an NSW-stage cp.async pipeline, so the activations are read once
// per CTA instead of once per vocab tile.  Warp (wr, wt) of the 4 x kLmWideWT warps takes tile rows
// 16 wr .. 16 wr + 15 and token blocks wt, wt + kLmWideWT, ...  Each lane keeps, per token, the best
// (value, lowest index) over the tiles it has seen; the CTA writes one partial per token to
// pval/pidx[blockIdx.x].
constexpr int kLmWideWT = 4;
template <int TBW, int NSW>
struct LmWide {
  static constexpr int BT = 8 * TBW;
  static constexpr int THREADS = kGemmThreads * kLmWideWT;
  static constexpr int TBP = (TBW + kLmWideWT - 1) / kLmWideWT;  // token blocks per warp
  static __host__ __device__ int xrow(int K) { return K + 8; }          // fp16 per staged token row
  static __host__ __device__ int wrow(int K) { return (K >> 1) + 16; }  // bytes per staged weight row
  static __host__ __device__ size_t stage(int K) {
    return ((size_t)kGemmRows * wrow(K) + (size_t)kGemmRows * (K >> 5) * 4 + 15) & ~(size_t)15;
  }
  static __host__ __device__ size_t smem(int K) { return (size_t)2 * BT * xrow(K) * 2 + NSW * stage(K); }
};

template <int TBW, int NSW>
__global__ void __launch_bounds__(LmWide<TBW, NSW>::THREADS, 1) lwe_gemm_lm_wide(const __grid_constant__ LweArgs a,
                                                                                 int T, int tiles_per_cta) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LmWide<TBW, NSW>;
  constexpr int BT = C::BT, NT = C::THREADS, TBP = C::TBP;
  __shared__ float bvs[4 * BT];
  __shared__ int bis[4 * BT];
  const int V = a.m.vocab, K = a.m.D, ng = K >> 5;
  const int XR = C::xrow(K), WR = C::wrow(K);
  const size_t wbytes = (size_t)kGemmRows * WR, stage = C::stage(K);
  __half* xh = reinterpret_cast<__half*>(smem);
  __half* xl = xh + (size_t)BT * XR;
  unsigned char* wst = reinterpret_cast<unsigned char*>(xl + (size_t)BT * XR);
  const int ntiles = (V + kGemmRows - 1) / kGemmRows;
  const int rt0 = blockIdx.x * tiles_per_cta, nt = max(0, min(ntiles, rt0 + tiles_per_cta) - rt0);
  const int t0 = blockIdx.y * BT;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gid = lane >> 2, t = lane & 3;
  const int wr = warp & 3, wt = warp >> 2;
  const uint8_t* W = reinterpret_cast<const uint8_t*>(a.m.lm.w);
  const float* S = a.m.lm.s;
  auto issue_w = [&](int rt, int st) {
    unsigned char* dst = wst + (size_t)st * stage;
    float* sdst = reinterpret_cast<float*>(dst + wbytes);
    const int r0 = rt * kGemmRows, cpr = K >> 5;  // 16-byte chunks per packed row
    for (int j = tid; j < kGemmRows * cpr; j += NT) {
      const int r = j / cpr, c = j % cpr, row = r0 + r;
      cp_async16(dst + r * WR + c * 16, W + (size_t)min(row, V - 1) * (K >> 1) + c * 16, row < V);
    }
    for (int j = tid; j < kGemmRows * ng; j += NT) {
      const int row = r0 + j / ng;
      cp_async4(sdst + j, S + (size_t)min(row, V - 1) * ng + j % ng, row < V);
    }
  };
  // weight stages first (no kernel writes them), then wait for the previous kernel, then activations
#pragma unroll
  for (int s = 0; s < NSW - 1; ++s) {
    if (s < nt) issue_w(rt0 + s, s);
    cp_async_commit();
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (a.skip && *a.skip) {  // a finished speculative loop replays as no-ops
    cp_async_wait<0>();
    return;
  }
  {
    const int cpx = K >> 3;  // 16-byte chunks per token row
    for (int j = tid; j < BT * cpx; j += NT) {
      const int r = j / cpx, c = j % cpx, tok = t0 + r;
      const size_t off = (size_t)min(tok, T - 1) * a.ldx + c * 8;
      cp_async16(xh + r * XR + c * 8, a.xh + off, tok < T);
      cp_async16(xl + r * XR + c * 8, a.xl + off, tok < T);
    }
    cp_async_commit();
  }
  // this warp's token blocks: b = wt + kLmWideWT * j, j < TBP (b < TBW)
  float bv[TBP][2];
  int bi[TBP][2];
#pragma unroll
  for (int j = 0; j < TBP; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      bv[j][e] = -INFINITY;
      bi[j][e] = 0x7fffffff;
    }
  const int ia = wr * 16 + gid, ib = ia + 8;
  for (int i = 0; i < nt; ++i) {
    if (i == 0) cp_async_wait<0>();
    else cp_async_wait<NSW - 2>();
    __syncthreads();  // tile i has landed everywhere; every warp is done with tile i - 1's stage
    {
      const int in = i + NSW - 1;
      if (in < nt) issue_w(rt0 + in, in % NSW);
      cp_async_commit();
    }
    const unsigned char* ws = wst + (size_t)(i % NSW) * stage;
    const float* ss = reinterpret_cast<const float*>(ws + wbytes);
    const uint32_t* wr0 = reinterpret_cast<const uint32_t*>(ws + ia * WR);
    const uint32_t* wr1 = reinterpret_cast<const uint32_t*>(ws + ib * WR);
    float acc[TBP][4];
#pragma unroll
    for (int j = 0; j < TBP; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int g = 0; g < ng; ++g) {
      uint32_t a0[4], a1[4];
      load_a_frag(wr0 + 4 * g, wr1 + 4 * g, 0, t, a0);
      load_a_frag(wr0 + 4 * g, wr1 + 4 * g, 1, t, a1);
      const float sc0 = ss[ia * ng + g], sc1 = ss[ib * ng + g];
#pragma unroll
      for (int j = 0; j < TBP; ++j) {
        const int b = wt + kLmWideWT * j;
        if (b >= TBW) break;
        const int xo = (b * 8 + (lane & 7)) * XR + g * 32 + (lane >> 3) * 8;
        uint32_t bh[4], bl[4];
        ldsm_x4(bh, xh + xo);
        ldsm_x4(bl, xl + xo);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(d, a0, bh[0], bh[1]);
        mma16816(d, a0, bl[0], bl[1]);
        mma16816(d, a1, bh[2], bh[3]);
        mma16816(d, a1, bl[2], bl[3]);
        acc[j][0] = fmaf(sc0, d[0], acc[j][0]);
        acc[j][1] = fmaf(sc0, d[1], acc[j][1]);
        acc[j][2] = fmaf(sc1, d[2], acc[j][2]);
        acc[j][3] = fmaf(sc1, d[3], acc[j][3]);
      }
    }
    // this tile's candidate per (token, lane): row ia, or ib when larger (ia < ib keeps ties)
    const int ra = (rt0 + i) * kGemmRows + ia, rb = ra + 8;
#pragma unroll
    for (int j = 0; j < TBP; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = -INFINITY;
        int idx = 0x7fffffff;
        if (ra < V) {
          v = acc[j][e];
          idx = ra;
        }
        if (rb < V && acc[j][2 + e] > v) {
          v = acc[j][2 + e];
          idx = rb;
        }
        if (v > bv[j][e] || (v == bv[j][e] && idx < bi[j][e])) {
          bv[j][e] = v;
          bi[j][e] = idx;
        }
      }
  }
  cp_async_wait<0>();
  // reduce over gid (lanes with the same t), then over the 4 row warps of each token block
#pragma unroll
  for (int j = 0; j < TBP; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int b = wt + kLmWideWT * j;
      if (b >= TBW) break;
      float v = bv[j][e];
      int idx = bi[j][e];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
          v = ov;
          idx = oi;
        }
      }
      if (gid == 0) {
        bvs[wr * BT + b * 8 + 2 * t + e] = v;
        bis[wr * BT + b * 8 + 2 * t + e] = idx;
      }
    }
  __syncthreads();
  for (int tl = tid; tl < BT; tl += NT) {
    const int tok = t0 + tl;
    if (tok >= T) continue;
    float v = bvs[tl];
    int idx = bis[tl];
    for (int w = 1; w < 4; ++w) {
      const float ov = bvs[w * BT + tl];
      const int oi = bis[w * BT + tl];
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    a.pval[(size_t)blockIdx.x * a.lm_cap + tok] = v;
    a.pidx[(size_t)blockIdx.x * a.lm_cap + tok] = idx;
  }
}

// Wide w1/w3 GEMM for long forwards (prefill chunks): the lm_head layout above applied to
// lwe_gemm_w13.  Each CTA keeps its 8*TBW token rows of the normalised input in shared memory and
// streams its run of 32-row tiles of (w1, w3) through an NSW-stage pipeline; staged row i is matrix
// row 8 (i / 16) + i % 8 of w1 (i % 16 < 8) or w3 (as RowsPaired), so lane (gid, t) of row warp wr holds
// the w1 and w3 sums of matrix row 8 wr + gid.  Epilogue of lwe_gemm_w13: SiLU(u) * v with the token's
// 1/RMS, as fp16 hi/lo into xh2/xl2.
template <int TBW, int NSW>
__global__ void __launch_bounds__(LmWide<TBW, NSW>::THREADS, 1) lwe_gemm_w13_wide(const __grid_constant__ LweArgs a,
                                                                                  int T, int l, int tiles_per_cta) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LmWide<TBW, NSW>;
  constexpr int BT = C::BT, NT = C::THREADS, TBP = C::TBP;
  __shared__ float sinv[BT];
  const LayerDev& L = a.m.layers[l];
  const int FF = a.m.FF, K = a.m.D, ng = K >> 5;
  const int XR = C::xrow(K), WR = C::wrow(K);
  const size_t wbytes = (size_t)kGemmRows * WR, stage = C::stage(K);
  __half* xh = reinterpret_cast<__half*>(smem);
  __half* xl = xh + (size_t)BT * XR;
  unsigned char* wst = reinterpret_cast<unsigned char*>(xl + (size_t)BT * XR);
  const int ntiles = (FF + 31) / 32;
  const int rt0 = blockIdx.x * tiles_per_cta, nt = max(0, min(ntiles, rt0 + tiles_per_cta) - rt0);
  const int t0 = blockIdx.y * BT;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gid = lane >> 2, t = lane & 3;
  const int wr = warp & 3, wt = warp >> 2;
  const uint8_t* W1 = reinterpret_cast<const uint8_t*>(L.w1.w);
  const uint8_t* W3 = reinterpret_cast<const uint8_t*>(L.w3.w);
  auto issue_w = [&](int rt, int st) {
    unsigned char* dst = wst + (size_t)st * stage;
    float* sdst = reinterpret_cast<float*>(dst + wbytes);
    const int cpr = K >> 5;  // 16-byte chunks per packed row
    for (int j = tid; j < kGemmRows * cpr; j += NT) {
      const int r = j / cpr, c = j % cpr, row = rt * 32 + (r >> 4) * 8 + (r & 7);
      cp_async16(dst + r * WR + c * 16, ((r & 8) ? W3 : W1) + (size_t)min(row, FF - 1) * (K >> 1) + c * 16,
                 row < FF);
    }
    for (int j = tid; j < kGemmRows * ng; j += NT) {
      const int r = j / ng, row = rt * 32 + (r >> 4) * 8 + (r & 7);
      cp_async4(sdst + j, ((r & 8) ? L.w3.s : L.w1.s) + (size_t)min(row, FF - 1) * ng + j % ng, row < FF);
    }
  };
#pragma unroll
  for (int s = 0; s < NSW - 1; ++s) {
    if (s < nt) issue_w(rt0 + s, s);
    cp_async_commit();
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (a.skip && *a.skip) {  // a finished speculative loop replays as no-ops
    cp_async_wait<0>();
    return;
  }
  {
    const int cpx = K >> 3;  // 16-byte chunks per token row
    for (int j = tid; j < BT * cpx; j += NT) {
      const int r = j / cpx, c = j % cpx, tok = t0 + r;
      const size_t off = (size_t)min(tok, T - 1) * a.ldx + c * 8;
      cp_async16(xh + r * XR + c * 8, a.xh + off, tok < T);
      cp_async16(xl + r * XR + c * 8, a.xl + off, tok < T);
    }
    cp_async_commit();
  }
  for (int i = tid; i < BT; i += NT) sinv[i] = a.fold && t0 + i < T ? fold_inv(a, t0 + i) : 1.f;
  const int ia = wr * 16 + gid, ib = ia + 8;
  for (int i = 0; i < nt; ++i) {
    if (i == 0) cp_async_wait<0>();
    else cp_async_wait<NSW - 2>();
    __syncthreads();  // tile i has landed everywhere; every warp is done with tile i - 1's stage
    {
      const int in = i + NSW - 1;
      if (in < nt) issue_w(rt0 + in, in % NSW);
      cp_async_commit();
    }
    const unsigned char* ws = wst + (size_t)(i % NSW) * stage;
    const float* ss = reinterpret_cast<const float*>(ws + wbytes);
    const uint32_t* wr0 = reinterpret_cast<const uint32_t*>(ws + ia * WR);
    const uint32_t* wr1 = reinterpret_cast<const uint32_t*>(ws + ib * WR);
    float acc[TBP][4];
#pragma unroll
    for (int j = 0; j < TBP; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
    for (int g = 0; g < ng; ++g) {
      uint32_t a0[4], a1[4];
      load_a_frag(wr0 + 4 * g, wr1 + 4 * g, 0, t, a0);
      load_a_frag(wr0 + 4 * g, wr1 + 4 * g, 1, t, a1);
      const float sc0 = ss[ia * ng + g], sc1 = ss[ib * ng + g];
#pragma unroll
      for (int j = 0; j < TBP; ++j) {
        const int b = wt + kLmWideWT * j;
        if (b >= TBW) break;
        const int xo = (b * 8 + (lane & 7)) * XR + g * 32 + (lane >> 3) * 8;
        uint32_t bh[4], bl[4];
        ldsm_x4(bh, xh + xo);
        ldsm_x4(bl, xl + xo);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(d, a0, bh[0], bh[1]);
        mma16816(d, a0, bl[0], bl[1]);
        mma16816(d, a1, bh[2], bh[3]);
        mma16816(d, a1, bl[2], bl[3]);
        acc[j][0] = fmaf(sc0, d[0], acc[j][0]);
        acc[j][1] = fmaf(sc0, d[1], acc[j][1]);
        acc[j][2] = fmaf(sc1, d[2], acc[j][2]);
        acc[j][3] = fmaf(sc1, d[3], acc[j][3]);
      }
    }
    // epilogue (engine/infer.js:178-183, 522-524)
    const int r = (rt0 + i) * 32 + wr * 8 + gid;
    if (r < FF) {
#pragma unroll
      for (int j = 0; j < TBP; ++j) {
        const int b = wt + kLmWideWT * j;
        if (b >= TBW) break;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tl = b * 8 + 2 * t + e, tok = t0 + tl;
          if (tok >= T) continue;
          const float iv = sinv[tl];
          const float u = acc[j][e] * iv, v = acc[j][2 + e] * iv;
          const size_t off = (size_t)tok * a.ldx2 + r;
          split_hi_lo((u / (1.f + expf(-u))) * v, a.xh2[off], a.xl2[off]);
        }
      }
    }
  }
  cp_async_wait<0>();
}

// lm_head GEMM over the T rows in xh/xl with a per-CTA argmax epilogue: for each token, the best
// (value, lowest index) over the CTA's 64 vocab rows goes to pval/pidx[blockIdx.x][t].  Optional
// logits store [t][V].
template <int TBW>
__global__ void __launch_bounds__(kGemmThreads) lwe_gemm_lm(const __grid_constant__ LweArgs a, int T, float* logits) {
  extern __shared__ __align__(16) unsigned char smem[];
  using C = LweTile<TBW, 1, true>;
  constexpr int kLweBT = C::BT;
  const int V = a.m.vocab, K = a.m.D;
  const int r0 = blockIdx.x * kGemmRows, t0 = blockIdx.y * kLweBT;
  float acc[TBW][4];
  const RowsLinear rows{reinterpret_cast<const uint8_t*>(a.m.lm.w), a.m.lm.s, V, r0, K >> 1, K >> 5};
  // waits for the previous kernel inside, after requesting the first weight stages
  if (!q4_gemm_core<TBW, C::NS, 1, decltype(rows), C::GPS, true>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc, a.skip))
    return;  // a finished speculative loop replays as no-ops
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int ra = r0 + warp * 16 + gid, rb = ra + 8;
  __syncthreads();  // the pipeline buffers are reused below
  float* bv = reinterpret_cast<float*>(smem);            // [4 warps][kLweBT]
  int* bi = reinterpret_cast<int*>(bv + 4 * kLweBT);     // [4 warps][kLweBT]
#pragma unroll
  for (int b = 0; b < TBW; ++b) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tl = b * 8 + 2 * t + e, tok = t0 + tl;
      float v = -INFINITY;
      int idx = 0x7fffffff;
      if (ra < V) {
        v = acc[b][e];
        idx = ra;
      }
      if (rb < V && acc[b][2 + e] > v) {  // ra < rb: ties keep ra
        v = acc[b][2 + e];
        idx = rb;
      }
      if (logits && tok < T) {
        if (ra < V) logits[(size_t)tok * V + ra] = acc[b][e];
        if (rb < V) logits[(size_t)tok * V + rb] = acc[b][2 + e];
      }
      // reduce over gid (lanes with the same t): xor 4, 8, 16
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
          v = ov;
          idx = oi;
        }
      }
      if (gid == 0) {
        bv[warp * kLweBT + tl] = v;
        bi[warp * kLweBT + tl] = idx;
      }
    }
  }
  __syncthreads();
  for (int tl = threadIdx.x; tl < kLweBT; tl += blockDim.x) {
    const int tok = t0 + tl;
    if (tok >= T) continue;
    float v = bv[tl];
    int idx = bi[tl];
    for (int w = 1; w < 4; ++w) {
      const float ov = bv[w * kLweBT + tl];
      const int oi = bi[w * kLweBT + tl];
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    a.pval[(size_t)blockIdx.x * a.lm_cap + tok] = v;
    a.pidx[(size_t)blockIdx.x * a.lm_cap + tok] = idx;
  }
}

// Per token: argmax over the row-block partials -> amax[t]; optional scatter of the result.
__global__ void lwe_argmax_reduce(const __grid_constant__ LweArgs a, int T, int nblk) {
  pdl_enter();
  if (a.skip && *a.skip) return;  // a finished speculative loop replays as no-ops
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float v = -INFINITY;
  int idx = 0x7fffffff;
  for (int b = lane; b < nblk; b += 32) {
    const float ov = a.pval[(size_t)b * a.lm_cap + t];
    const int oi = a.pidx[(size_t)b * a.lm_cap + t];
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  if (lane == 0) a.amax[t] = idx;
}

// lm_head + argmax partials on the tcgen05 tile (tc5.cuh) for many rows without logits (a batched decode
// step): CTA (b, y) holds vocab rows 128 b .. + 127 against lm rows N y .. + N - 1 of the tiled final-norm
// output (xh3 / xl3, lwe_norm_split<true>) and writes, per lm row, the best (value, index) over its 128
// vocab rows to pval / pidx[b] (ties keep the lower index, as lwe_gemm_lm).  In each warp, a butterfly
// of xor-shuffles folds 32 rows x 16 tokens down to one token per lane pair (16 shuffles for 16
// tokens); the four warps of a column half then merge through shared memory.
__device__ __forceinline__ bool lm_better(float ov, int oi, float v, int i) { return ov > v || (ov == v && oi < i); }
template <int NV>
__device__ __forceinline__ void lm_fold(float (&v)[16], int (&ix)[16], int o, int lane) {
  const bool up = (lane & o) != 0;  // this lane keeps entries NV .. 2NV - 1, its partner 0 .. NV - 1
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float kv = up ? v[NV + i] : v[i], sv = up ? v[i] : v[NV + i];
    const int ki = up ? ix[NV + i] : ix[i], si = up ? ix[i] : ix[NV + i];
    const float ov = __shfl_xor_sync(0xffffffffu, sv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, si, o);
    const bool take = lm_better(ov, oi, kv, ki);
    v[i] = take ? ov : kv;
    ix[i] = take ? oi : ki;
  }
}

template <int N, int S>
__global__ void __launch_bounds__(tc5::kTc5Threads + 64, 1) lwe_lm_tc5(const __grid_constant__ LweArgs a, int T) {
  using namespace tc5;
  static_assert(N >= 32, "two column halves of 16-token chunks");
  extern __shared__ __align__(128) uint8_t smem[];
  const int V = a.m.vocab, K = a.m.D;
  const int r0 = blockIdx.x * kTc5Rows, t0 = blockIdx.y * N;
  // the copy thread waits for the final norm (griddepcontrol.wait) before its first activation copy
  const Tc5Acc acc = tc5_tile<N, S>(reinterpret_cast<const uint8_t*>(a.m.lm.w), a.m.lm.s, a.xh3, a.xl3, V, K,
                                    (T + 7) / 8, r0, t0, smem, true, a.err);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* bv = reinterpret_cast<float*>(smem);  // [4 row quarters][N] (the stages are idle now)
  int* bi = reinterpret_cast<int*>(bv + 4 * N);
  if (acc.ok && warp < kTc5Threads / 32) {
    const int cbeg = (warp >> 2) * (N / 2), q = warp & 3;
    const int row = r0 + q * 32 + lane;
    // the token of the 16-chunk this lane holds after the folds
    const int tk = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
    for (int c0 = cbeg; c0 < cbeg + N / 2; c0 += 16) {
      float v[16];
      int ix[16];
      tc5_cols16<N>(acc, warp, c0, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        ix[i] = row < V ? row : 0x7fffffff;
        if (row >= V) v[i] = -INFINITY;
      }
      lm_fold<8>(v, ix, 16, lane);
      lm_fold<4>(v, ix, 8, lane);
      lm_fold<2>(v, ix, 4, lane);
      lm_fold<1>(v, ix, 2, lane);
      const float ov = __shfl_xor_sync(0xffffffffu, v[0], 1);
      const int oi = __shfl_xor_sync(0xffffffffu, ix[0], 1);
      if (lm_better(ov, oi, v[0], ix[0])) {
        v[0] = ov;
        ix[0] = oi;
      }
      if ((lane & 1) == 0) {
        bv[q * N + c0 + tk] = v[0];
        bi[q * N + c0 + tk] = ix[0];
      }
    }
  }
  __syncthreads();
  if (acc.ok) {
    for (int c = threadIdx.x; c < N; c += blockDim.x) {
      const int t = t0 + c;
      if (t >= T) continue;
      float v = bv[c];
      int ix = bi[c];
#pragma unroll
      for (int q = 1; q < 4; ++q)
        if (lm_better(bv[q * N + c], bi[q * N + c], v, ix)) {
          v = bv[q * N + c];
          ix = bi[q * N + c];
        }
      a.pval[(size_t)blockIdx.x * a.lm_cap + t] = v;
      a.pidx[(size_t)blockIdx.x * a.lm_cap + t] = ix;
    }
  }
  tc5_release<N>(acc);
}

// ---------------------------------------------------------------------------------------------
// Layer GEMMs of a llama forward on the tcgen05 tile (tc5.cuh), fed by the load-time group images of the
// matrix (tc5_tile_pre).
// grid (row tiles, ceil(T / N), kz): CTA (b, y, z) multiplies 128 tile rows by tokens N y .. N y + N - 1
// over its share of the K groups (split-K when kz > 1: each CTA leaves its fp32 partial tile in
// a.skws, the last one of a tile (counter a.skctr) adds them in split order and runs the epilogue).
//   kTc5Qkv:   qkv[t][r] = acc / RMS_t + bias[r]                                (lwe_gemm_qkv, no RoPE)
//   kTc5Resid: x[t][r] += acc + bias[r]; with gn the next norm's x * gn as tiled fp16 hi/lo in nh/nl and
//              the 64-row halves' sums of squares of x in a.ss                   (lwe_gemm_resid)
//   kTc5W13:   w1/w3 pairs (Tc5Paired), xh2/xl2 tiled = SiLU(u / RMS) (v / RMS)  (lwe_gemm_w13)
// Every thread waits for the previous kernel (griddepcontrol.wait) before the epilogue touches a buffer
// another kernel writes; the producers only read weights before it.
enum Tc5Epi { kTc5Qkv = 0, kTc5Resid = 1, kTc5W13 = 2 };

// The 16 values of a lane (one tile row, 16 tokens) summed over the warp's 32 rows by a butterfly of
// xor-shuffles, in a fixed order: afterwards lanes 2i and 2i + 1 hold the sum of value
// tc5_fold_token(2i).
__device__ __forceinline__ float tc5_fold_sum(float (&v)[16], int lane) {
#pragma unroll
  for (int o = 16, nv = 8; o >= 2; o >>= 1, nv >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i >= nv) break;
      const float keep = up ? v[nv + i] : v[i], send = up ? v[i] : v[nv + i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}
__device__ __forceinline__ int tc5_fold_token(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

template <int N, int S, int EPI>
__global__ void __launch_bounds__(tc5::kTc5Threads + 64, 1)
    lwe_tc5_gemm(const __grid_constant__ LweArgs a, int T, Q4 w, Q4 w3, const float* bias, int R, int K,
                 const __half* xh, const __half* xl, const float* gn, __half* nh, __half* nl, Tc5Pre pre) {
  using namespace tc5;
  static_assert(N >= 32 && N % 32 == 0, "two column halves of 16-token chunks");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float sinv[N];
  __shared__ float ssq[4][N];
  __shared__ int last;
  const int NG = K / 32, kz = gridDim.z, z = blockIdx.z;
  const int ngz = (NG + kz - 1) / kz, g0 = z * ngz, ng = min(ngz, NG - g0);
  const int t0 = blockIdx.y * N, T8 = (T + 7) / 8;
  // the tokens' 1/RMS (from the previous kernel's sums of squares), staged by the copy warp's spare
  // lanes while the K loop runs
  auto side = [&](int lane) {
    if (EPI != kTc5Resid)
      for (int i = lane - 1; i < N; i += 31) sinv[i] = t0 + i < T ? fold_inv(a, t0 + i) : 1.f;
  };
  // the matrix's group images from the load-time expansion (the Q4 pointers w / w3 are not read here)
  const Tc5Acc acc = tc5_tile_pre<N, S>(pre.img + ((size_t)blockIdx.x * NG + g0) * kTc5GroupImage,
                                        pre.down[blockIdx.x], xh, xl, T8, t0, g0, ng, smem, true, a.err, side);
  pdl_enter();  // the previous kernel's x, ss and activation buffers are complete
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool epi_warp = warp < kTc5Threads / 32;
  const int q = warp & 3, cbeg = (warp >> 2) * (N / 2);
  const int tile = blockIdx.y * gridDim.x + blockIdx.x;
  // split-K: this CTA's partial tile [N columns][128 rows] in the workspace, then the last CTA sums them
  bool run = acc.ok;
  if (kz > 1) {
    float* mine = a.skws + ((size_t)tile * kz + z) * kTc5Rows * N;
    if (acc.ok && epi_warp)
      for (int c0 = cbeg; c0 < cbeg + N / 2; c0 += 16) {
        float v[16];
        tc5_cols16<N>(acc, warp, c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) __stcg(mine + (size_t)(c0 + i) * kTc5Rows + q * 32 + lane, v[i]);
      }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int done = atomicAdd(&a.skctr[tile], 1) + 1;
      last = done == kz;
      if (last) a.skctr[tile] = 0;
    }
    __syncthreads();
    run = run && last;
    if (run) __threadfence();
  }
  if (run && epi_warp) {
    for (int c0 = cbeg; c0 < cbeg + N / 2; c0 += 16) {
      float v[16];
      if (kz > 1) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0.f;
        for (int zz = 0; zz < kz; ++zz) {
          const float* p = a.skws + ((size_t)tile * kz + zz) * kTc5Rows * N + q * 32 + lane;
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] += __ldcg(p + (size_t)(c0 + i) * kTc5Rows);
        }
      } else {
        tc5_cols16<N>(acc, warp, c0, v);
      }
      if constexpr (EPI == kTc5Qkv) {
        const int r = blockIdx.x * kTc5Rows + q * 32 + lane;
        if (r < R) {
          const float b = bias ? bias[r] : 0.f;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = t0 + c0 + i;
            if (t < T) {
              const float y = v[i] * sinv[c0 + i];
              a.qkv[(size_t)t * R + r] = bias ? y + b : y;
            }
          }
        }
      } else if constexpr (EPI == kTc5Resid) {
        const int r = blockIdx.x * kTc5Rows + q * 32 + lane;
        const float b = bias && r < R ? bias[r] : 0.f, gr = gn && r < R ? gn[r] : 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = t0 + c0 + i;
          float sq = 0.f;
          if (t < T && r < R) {
            float* px = a.x + (size_t)t * R + r;
            const float xn = *px + (bias ? v[i] + b : v[i]);
            *px = xn;
            if (gn) {
              const size_t o = tiled_at(t, r, T8);
              split_hi_lo(xn * gr, nh[o], nl[o]);
              sq = xn * xn;
            }
          }
          v[i] = sq;
        }
        if (gn) {
          const float s2 = tc5_fold_sum(v, lane);
          if ((lane & 1) == 0) ssq[q][c0 + tc5_fold_token(lane)] = s2;
        }
      } else {  // kTc5W13: lane j < 16 holds u of FF row f, lane j + 16 holds v of the same row
        const bool up = lane >= 16;
        const int f = blockIdx.x * 64 + 16 * q + (lane & 15);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float other = __shfl_xor_sync(0xffffffffu, up ? v[i] : v[8 + i], 16);
          const int c = c0 + (up ? 8 + i : i), t = t0 + c;
          const float iv = sinv[c];
          const float u = (up ? other : v[i]) * iv, g = (up ? v[8 + i] : other) * iv;
          if (t < T && f < R) {
            const size_t o = tiled_at(t, f, T8);
            split_hi_lo((u / (1.f + expf(-u))) * g, a.xh2[o], a.xl2[o]);
          }
        }
      }
    }
  }
  if (EPI == kTc5Resid && gn) {
    __syncthreads();
    if (run)
      for (int i = tid; i < N; i += blockDim.x) {
        const int t = t0 + i;
        if (t >= T) continue;
        float* ps = a.ss + (size_t)t * kLweSsStride + 2 * blockIdx.x;
        ps[0] = ssq[0][i] + ssq[1][i];  // rows 0 .. 63 of the tile
        if (2 * blockIdx.x + 1 < kLweSsStride) ps[1] = ssq[2][i] + ssq[3][i];
      }
  }
  tc5_release<N>(acc);
}

// One greedy step of the replicated multi-sequence decode for every active slot: record the new id,
// apply the stop rules of engine/infer.js:617-639 and advance token and position.
__global__ void lwe_decode_advance(const __grid_constant__ LweArgs a, int T, int max_new, int eos,
                                   int32_t* out_ids, int32_t* counts, const int32_t* prompt_len) {
  pdl_enter();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  if (counts[t] < 0) return;  // finished (sign flipped)
  const int id = a.amax[t];
  const int n = counts[t];
  out_ids[(size_t)t * max_new + n] = id;
  const int nn = n + 1;
  const bool stop = id == eos || nn >= max_new || prompt_len[t] + nn >= a.m.kv_len;
  counts[t] = stop ? -nn : nn;
  a.tok[t] = id;
  a.pos[t] = prompt_len[t] + nn - 1;
}

__global__ void lwe_mark(int32_t* status, int idx) {
  const uint64_t t = globaltimer();
  status[idx] = (int32_t)(uint32_t)t;
  status[idx + 1] = (int32_t)(uint32_t)(t >> 32);
}

// First id of a generate from the prefill's argmax (engine/infer.js:611-623).
__global__ void lwe_first_token(const int32_t* amax, int32_t* out_ids, int32_t* status, int eos, int forwards,
                                int32_t* stream) {
  const int id = amax[0];
  out_ids[0] = id;
  stream_publish(stream, 0, id, 0);
  status[ST_NGEN] = 1;
  status[ST_STOP] = id == eos ? 0 : 1;
  status[ST_FORWARDS] = forwards;
  const uint64_t t = globaltimer();
  status[ST_TFIRST] = (int32_t)(uint32_t)t;
  status[ST_TFIRST + 1] = (int32_t)(uint32_t)(t >> 32);
  status[ST_TEND] = (int32_t)(uint32_t)t;
  status[ST_TEND + 1] = (int32_t)(uint32_t)(t >> 32);
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------
// Tokens per CTA: for T < 512, the largest tile that still gives two CTAs per SM, else the smallest.
// (A 27-point sweep of forced tiles and k splits on the 256-row decode step found none better.)
static int pick_tbw(int row_tiles, int T) {
  // Long prefill chunks: the smallest tile everywhere (thousands of CTAs) measured 10 % faster than
  // the larger tiles on 1,024-token chunks; a 256-row decode step keeps the rule below.
  if (T >= 512) return 2;
  constexpr int kTarget = 2 * 148;
  if (T <= 16) return 2;  // one token tile either way: the smallest wastes the least
  if (T <= 32) return row_tiles >= kTarget ? 4 : 2;
  if ((long)row_tiles * ((T + 63) / 64) >= kTarget) return 8;
  if ((long)row_tiles * ((T + 31) / 32) >= kTarget) return 4;
  return 2;
}

// Tokens per CTA as above; then the in-CTA k split for GEMMs that still have few CTAs, and for very
// few CTAs (a handful of tokens) a split of the k groups across CTAs as well (at least 8 groups each).
static int pick_ks(int ctas) {
  return ctas >= 2 * 148 ? 1 : (ctas >= 148 ? 2 : 4);
}
static int pick_ksplit(int ctas, int K, int TBW) {
  if (ctas >= 96) return 1;  // enough CTAs with the in-CTA split alone
  int z = (2 * 148 + ctas - 1) / ctas;
  z = std::min(z, std::max(1, (K / 32) / 8));
  z = std::min(z, 16);
  // the partial tiles must fit the workspace
  while (z > 1 && (size_t)ctas * z * kGemmThreads * TBW * 4 * 4 > kLweSplitKBytes) --z;
  return z;
}

// MLLM_LWE_DEBUG=1: report the first failing launch on stderr (kernel, tile, k split, grid).
static void lwe_debug_check(const char* what, int tb, int ks, int tiles, int T, int kz, size_t smem) {
  static const bool on = getenv("MLLM_LWE_DEBUG") != nullptr;
  if (!on) return;
  const cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess)
    fprintf(stderr, "lwe launch %s<%d,%d> tiles %d T %d kz %d smem %zu: %s\n", what, tb, ks, tiles, T, kz, smem,
            cudaGetErrorString(e));
}
#define LWE_LAUNCH_(KER, TB, KSV, TILES, T, KZ, ...)                                                  \
  lwe_launch(KER<TB, KSV>, dim3(TILES, ((T) + 8 * TB - 1) / (8 * TB), KZ), dim3(LweTile<TB, KSV>::THREADS), \
             LweTile<TB, KSV>::smem(), st, __VA_ARGS__);                                              \
  lwe_debug_check(#KER, TB, KSV, TILES, T, KZ, LweTile<TB, KSV>::smem())
#define LWE_GEMM(KER, ROWS_PER_CTA, R, K, T, ...)                                                     \
  do {                                                                                                \
    const int _tiles = ((R) + (ROWS_PER_CTA)-1) / (ROWS_PER_CTA);                                     \
    const int _tbw = pick_tbw(_tiles, (T));                                                           \
    const int _ctas = _tiles * (((T) + 8 * _tbw - 1) / (8 * _tbw));                                   \
    const int _ks = pick_ks(_ctas);                                                                   \
    const int _kz = pick_ksplit(_ctas, (K), _tbw);                                                    \
    switch (_tbw * 8 + _ks) {                                                                         \
      case 65: LWE_LAUNCH_(KER, 8, 1, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 66: LWE_LAUNCH_(KER, 8, 2, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 68: LWE_LAUNCH_(KER, 8, 4, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 33: LWE_LAUNCH_(KER, 4, 1, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 34: LWE_LAUNCH_(KER, 4, 2, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 36: LWE_LAUNCH_(KER, 4, 4, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 17: LWE_LAUNCH_(KER, 2, 1, _tiles, T, _kz, __VA_ARGS__); break;                            \
      case 18: LWE_LAUNCH_(KER, 2, 2, _tiles, T, _kz, __VA_ARGS__); break;                            \
      default: LWE_LAUNCH_(KER, 2, 4, _tiles, T, _kz, __VA_ARGS__); break;                            \
    }                                                                                                 \
  } while (0)
#define LWE_GEMM_LM(R, T, ...)                                                                        \
  do {                                                                                                \
    const int _tiles = ((R) + kGemmRows - 1) / kGemmRows;                                             \
    switch (pick_tbw(_tiles, (T))) {                                                                  \
      case 8: lwe_launch(lwe_gemm_lm<8>, dim3(_tiles, ((T) + 63) / 64), dim3(kGemmThreads), LweTile<8, 1, true>::smem(), st, __VA_ARGS__); break; \
      case 4: lwe_launch(lwe_gemm_lm<4>, dim3(_tiles, ((T) + 31) / 32), dim3(kGemmThreads), LweTile<4, 1, true>::smem(), st, __VA_ARGS__); break; \
      default: lwe_launch(lwe_gemm_lm<2>, dim3(_tiles, ((T) + 15) / 16), dim3(kGemmThreads), LweTile<2, 1, true>::smem(), st, __VA_ARGS__); \
    }                                                                                                 \
  } while (0)

template <class F>
static cudaError_t smem_attr(F* f, size_t bytes) {
  // always set: the kernels' static shared memory counts against the 48 KB default as well
  return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}
template <int TBW, int KS>
static cudaError_t gemm_attrs_ks() {
  const size_t b = LweTile<TBW, KS>::smem();
  cudaError_t e = smem_attr(lwe_gemm_qkv<TBW, KS>, b);
  if (e == cudaSuccess) e = smem_attr(lwe_gemm_resid<TBW, KS>, b);
  if (e == cudaSuccess) e = smem_attr(lwe_gemm_w13<TBW, KS>, b);
  if (e == cudaSuccess) e = smem_attr(lwe_gemm_fc<TBW, KS>, b);
  return e;
}
template <int TBW>
static cudaError_t gemm_attrs() {
  cudaError_t e = gemm_attrs_ks<TBW, 1>();
  if (e == cudaSuccess) e = gemm_attrs_ks<TBW, 2>();
  if (e == cudaSuccess) e = gemm_attrs_ks<TBW, 4>();
  if (e == cudaSuccess) e = smem_attr(lwe_gemm_lm<TBW>, LweTile<TBW, 1, true>::smem());
  return e;
}

template <bool F>
static void launch_attention_split(const LweArgs& a, const LweHost& h, int T, cudaStream_t st) {
  const int rep = a.m.NH / a.m.NKV;
  int chunk, S;
  lwe_attn_split_shape(a.m.kv_len, &chunk, &S);
  const dim3 grid(T, a.m.NKV, S);
  const size_t sm = (size_t)2 * kAttnChunk * 64 * 4;
  switch (rep) {
    case 1: lwe_launch(lwe_attn_split<1, F>, grid, dim3(64), sm, st, a, T, h.attn_part, h.attn_ctr); break;
    case 2: lwe_launch(lwe_attn_split<2, F>, grid, dim3(64), sm, st, a, T, h.attn_part, h.attn_ctr); break;
    case 3: lwe_launch(lwe_attn_split<3, F>, grid, dim3(64), sm, st, a, T, h.attn_part, h.attn_ctr); break;
    default: lwe_launch(lwe_attn_split<4, F>, grid, dim3(64), sm, st, a, T, h.attn_part, h.attn_ctr); break;
  }
}

template <bool F>
static void launch_attention_t(const LweArgs& a, int T, cudaStream_t st) {
  const int rep = a.m.NH / a.m.NKV;
  const dim3 grid(T, a.m.NKV);
  const size_t sm = attention_smem(rep, a.m.kv_len);
  switch (rep) {
    case 1: lwe_launch(lwe_attention<1, F>, grid, dim3(kAttnThreads), sm, st, a, T); break;
    case 2: lwe_launch(lwe_attention<2, F>, grid, dim3(kAttnThreads), sm, st, a, T); break;
    case 3: lwe_launch(lwe_attention<3, F>, grid, dim3(kAttnThreads), sm, st, a, T); break;
    default: lwe_launch(lwe_attention<4, F>, grid, dim3(kAttnThreads), sm, st, a, T); break;
  }
}

template <bool F>
static cudaError_t attention_attr(int need) {
  cudaError_t e = cudaFuncSetAttribute(lwe_attention<1, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(lwe_attention<2, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(lwe_attention<3, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(lwe_attention<4, F>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  return e;
}

// Wide lm_head GEMM (no logits): the largest token tile / pipeline depth whose shared memory fits.
static int g_lm_wide_cap = 0;  // dynamic shared memory granted to lwe_gemm_lm_wide (0: not set up)
template <int TBW, int NSW>
static bool try_lm_wide(const LweArgs& a, int T, cudaStream_t st, int sms, int* nblk) {
  using C = LmWide<TBW, NSW>;
  const size_t sm = C::smem(a.m.D);
  if (sm > (size_t)g_lm_wide_cap) return false;
  const int tiles = (a.m.vocab + kGemmRows - 1) / kGemmRows;
  const int tt = (T + C::BT - 1) / C::BT;
  int g = std::max(1, sms / tt);
  const int tpc = (tiles + g - 1) / g;
  g = (tiles + tpc - 1) / tpc;
  lwe_launch(lwe_gemm_lm_wide<TBW, NSW>, dim3(g, tt), dim3(C::THREADS), sm, st, a, T, tpc);
  *nblk = g;
  return true;
}
static bool launch_lm_wide(const LweArgs& a, int T, cudaStream_t st, int* nblk) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  return try_lm_wide<8, 3>(a, T, st, sms, nblk) || try_lm_wide<4, 3>(a, T, st, sms, nblk) ||
         try_lm_wide<4, 2>(a, T, st, sms, nblk) || try_lm_wide<2, 2>(a, T, st, sms, nblk);
}

// lm_head on the tcgen05 tile: the final norm writes the tiled halves, then one CTA per 128 vocab rows
// and N lm rows; the partials are one per vocab tile.
static bool g_lm_tc5_ok = false;  // shared-memory attributes granted (lwe_setup)
static void launch_lm_tc5(const LweArgs& a, int T, const float* norm_f, const int* src, cudaStream_t st, int* nblk) {
  lwe_launch(lwe_norm_split<true>, dim3(T), dim3(128), 0, st, a, T, norm_f, src);
  const int tiles = (a.m.vocab + tc5::kTc5Rows - 1) / tc5::kTc5Rows;
  constexpr int kThreads = tc5::kTc5Threads + 64;
  if (T > 128)
    lwe_launch(lwe_lm_tc5<256, 4>, dim3(tiles, (T + 255) / 256), dim3(kThreads), tc5::tc5_smem_bytes<256, 4>(), st, a,
               T);
  else
    lwe_launch(lwe_lm_tc5<128, 6>, dim3(tiles, (T + 127) / 128), dim3(kThreads), tc5::tc5_smem_bytes<128, 6>(), st,
               a, T);
  *nblk = tiles;
}

// Layer GEMMs on the tcgen05 tile (lwe_tc5_gemm).  Tokens per CTA: 32 while that grid fits one wave of
// the SMs or the 64-token tile's resident activations would not fit, else 64.  The K groups are split
// over several CTAs as far as the resident activations need to fit, and further (up to 4) while the
// grid stays within one wave and each CTA keeps >= 12 groups.
constexpr int kTc5PreStages = 4;  // stages of one group image
static int g_tc5_gemm_cap = 0;  // dynamic shared memory granted to lwe_tc5_gemm (0: not set up)
static int g_sms = 0;
template <int N, int EPI>
static void tc5_gemm_attr() {
  if (smem_attr(lwe_tc5_gemm<N, kTc5PreStages, EPI>, g_tc5_gemm_cap) != cudaSuccess) {
    (void)cudaGetLastError();
    g_tc5_gemm_cap = 0;
  }
}
int tc5_pre_tiles(int R, bool paired) { return paired ? (R + 63) / 64 : (R + tc5::kTc5Rows - 1) / tc5::kTc5Rows; }
size_t tc5_pre_bytes(int R, int K, bool paired) {
  return (size_t)tc5_pre_tiles(R, paired) * (K / 32) * tc5::kTc5GroupImage;
}
cudaError_t tc5_expand(const Q4& w, const Q4* w3, int R, int K, const Tc5Pre& p, cudaStream_t st) {
  using namespace tc5;
  const dim3 grid(tc5_pre_tiles(R, w3 != nullptr), K / 32);
  if (w3)
    tc5_expand_kernel<<<grid, 256, 0, st>>>(Tc5Paired{reinterpret_cast<const uint8_t*>(w.w), w.s,
                                                      reinterpret_cast<const uint8_t*>(w3->w), w3->s, R, K, 0},
                                            K / 32, p.img, p.down);
  else
    tc5_expand_kernel<<<grid, 256, 0, st>>>(Tc5Linear{reinterpret_cast<const uint8_t*>(w.w), w.s, R, K, 0}, K / 32,
                                            p.img, p.down);
  return cudaGetLastError();
}
struct Tc5Shape {
  int N, tt, kz, ngz;
  size_t smem;
};
static bool tc5_gemm_shape(int T, int rtiles, int K, Tc5Shape* sh) {
  using namespace tc5;
  if (g_tc5_gemm_cap <= 0 || K % 32) return false;
  const int NG = K / 32, sms = g_sms > 0 ? g_sms : 148;
  // shared memory (tc5_smem_pre): the image ring and the alignment slack, then N x 128 bytes of
  // activation halves per group
  const int fixed = kTc5PreStages * kTc5GroupImage + 1024;
  auto max_groups = [&](int n) { return (g_tc5_gemm_cap - fixed) / (n * 128); };
  // 64-token tiles only where the 32-token grid would take more than one wave and no K split is needed
  const int N = (long)rtiles * ((T + 31) / 32) <= sms || NG > max_groups(64) ? 32 : 64;
  const int tt = (T + N - 1) / N, tiles = rtiles * tt;
  const int maxg = max_groups(N);
  if (maxg < 1) return false;
  int kz = (NG + maxg - 1) / maxg;
  while (kz < 4 && (long)tiles * (kz + 1) <= sms && NG / (kz + 1) >= 12) ++kz;
  const int ngz = (NG + kz - 1) / kz;
  kz = (NG + ngz - 1) / ngz;  // every split keeps at least one group
  if (kz > 1 && (tiles > kLweSplitKTiles || (size_t)tiles * kz * kTc5Rows * N * 4 > kLweSkwsBytes)) return false;
  const size_t sm = tc5_smem_pre(N, kTc5PreStages, ngz);
  if (sm > (size_t)g_tc5_gemm_cap) return false;
  *sh = Tc5Shape{N, tt, kz, ngz, sm};
  return true;
}
// Whether every layer GEMM of a T-row llama forward has a tcgen05 shape (all of them must: the forward's
// GEMM inputs are then tiled).
static bool tc5_gemms_fit(const ModelDev& md, int T) {
  Tc5Shape sh;
  const int dt = (md.D + tc5::kTc5Rows - 1) / tc5::kTc5Rows;
  return tc5_gemm_shape(T, (md.QKV + tc5::kTc5Rows - 1) / tc5::kTc5Rows, md.D, &sh) &&
         tc5_gemm_shape(T, dt, md.D, &sh) && tc5_gemm_shape(T, (md.FF + 63) / 64, md.D, &sh) &&
         tc5_gemm_shape(T, dt, md.FF, &sh);
}
template <int EPI>
static void launch_tc5_gemm(const LweArgs& a, int T, int rtiles, int R, int K, Q4 w, Q4 w3, const float* bias,
                            const __half* xh, const __half* xl, const float* gn, __half* nh, __half* nl,
                            const Tc5Pre& pre, cudaStream_t st) {
  Tc5Shape sh;
  (void)tc5_gemm_shape(T, rtiles, K, &sh);  // tc5_gemms_fit checked it for the forward
  const dim3 grid(rtiles, sh.tt, sh.kz), block(tc5::kTc5Threads + 64);
  if (sh.N == 32)
    lwe_launch(lwe_tc5_gemm<32, kTc5PreStages, EPI>, grid, block, sh.smem, st, a, T, w, w3, bias, R, K, xh, xl, gn, nh,
               nl, pre);
  else
    lwe_launch(lwe_tc5_gemm<64, kTc5PreStages, EPI>, grid, block, sh.smem, st, a, T, w, w3, bias, R, K, xh, xl, gn, nh,
               nl, pre);
  lwe_debug_check("lwe_tc5_gemm", sh.N, EPI, rtiles, T, sh.kz, sh.smem);
}

// Wide w1/w3 GEMM for long forwards (K must fit the 64-token tile; else the per-tile GEMM).
static bool launch_w13_wide(const LweArgs& a, int T, int l, cudaStream_t st) {
  using C = LmWide<8, 3>;
  const size_t sm = C::smem(a.m.D);
  if (sm > (size_t)g_lm_wide_cap) return false;
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  const int tiles = (a.m.FF + 31) / 32, tt = (T + C::BT - 1) / C::BT;
  int g = std::max(1, sms / tt);
  const int tpc = (tiles + g - 1) / g;
  g = (tiles + tpc - 1) / tpc;
  lwe_launch(lwe_gemm_w13_wide<8, 3>, dim3(g, tt), dim3(C::THREADS), sm, st, a, T, l, tpc);
  return true;
}

// One-time kernel attributes: the attention's shared memory grows with kv_len.
cudaError_t lwe_setup(int kv_len) {
  {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    const int cap = optin - 4096;  // room for the kernel's static reduction arrays
    if (smem_attr(lwe_gemm_lm_wide<8, 3>, cap) == cudaSuccess && smem_attr(lwe_gemm_lm_wide<4, 3>, cap) == cudaSuccess &&
        smem_attr(lwe_gemm_lm_wide<4, 2>, cap) == cudaSuccess && smem_attr(lwe_gemm_lm_wide<2, 2>, cap) == cudaSuccess &&
        smem_attr(lwe_gemm_w13_wide<8, 3>, cap) == cudaSuccess)
      g_lm_wide_cap = cap;
    else
      (void)cudaGetLastError();
  }
  {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    g_tc5_gemm_cap = optin - 4096;  // room for the kernel's static arrays
    tc5_gemm_attr<32, kTc5Qkv>();
    tc5_gemm_attr<32, kTc5Resid>();
    tc5_gemm_attr<32, kTc5W13>();
    tc5_gemm_attr<64, kTc5Qkv>();
    tc5_gemm_attr<64, kTc5Resid>();
    tc5_gemm_attr<64, kTc5W13>();
  }
  g_lm_tc5_ok = smem_attr(lwe_lm_tc5<256, 4>, (int)tc5::tc5_smem_bytes<256, 4>()) == cudaSuccess &&
                smem_attr(lwe_lm_tc5<128, 6>, (int)tc5::tc5_smem_bytes<128, 6>()) == cudaSuccess;
  if (!g_lm_tc5_ok) (void)cudaGetLastError();
  cudaError_t e = gemm_attrs<2>();
  if (e == cudaSuccess) e = gemm_attrs<4>();
  if (e == cudaSuccess) e = gemm_attrs<8>();
  if (e != cudaSuccess) return e;
  const int need = (int)attention_smem(kLweMaxRep, kv_len);
  e = attention_attr<false>(need);
  return e == cudaSuccess ? attention_attr<true>(need) : e;
}

// A forward over T tokens whose ids/slots/positions are already in a.tok/a.slot/a.pos.  When
// lm_T > 0 the lm_head runs on lm_T rows — the token rows a.lm_src[0..lm_T) when lm_from_src, else
// rows 0..lm_T — and leaves the argmax per row in a.amax; logits (nullable) receives [lm_T][V].
cudaError_t lwe_forward(LweArgs a, const LweHost& h, int T, int lm_T, bool lm_from_src, float* logits,
                        bool one_per_slot, cudaStream_t st) {
  const ModelDev& md = a.m;
  const int nl = md.n_layers;
  // RMSNorm folded into the GEMMs (llama): the residual GEMMs write x * gain and sums of squares,
  // the consumers apply 1/RMS.  LayerNorm (GPT-2) keeps separate norm kernels.
  const bool fold = md.arch == 0 && h.fold_norm;
  a.fold = fold ? 1 : 0;
  // llama forwards of many rows: every layer GEMM on the tcgen05 tile, GEMM inputs in the tiled layout
  // (the matrices were expanded into the tile's group images at load when MLLM_LWE_GEMM_TC5 is set)
  const bool tc = fold && h.gemm_tc5 && (int)h.pre.size() == nl * kPreMats && T >= kTc5GemmRows && !a.skip &&
                  tc5_gemms_fit(md, T);
  a.tiled = tc ? 1 : 0;
  g_lwe_pdl = h.pdl != 0;
  lwe_launch(lwe_embed, dim3(T), dim3(128), 0, st, a, T, h.layers[0].norm1);  // + norm1 of layer 0
  for (int l = 0; l < nl; ++l) {
    const LayerDev& L = h.layers[l];
    a.layer = l;
    // A few rows (a verify forward): RoPE and the K/V cache rows in the QKV epilogue.  Long forwards keep
    // lwe_rope_kv (the staged epilogue measured 2-3 % slower on 512- and 1,024-token prefill), and the
    // batched decode step's attention does them itself.
    const bool rope_epi = !one_per_slot && h.rope_epi && T <= kLweSplitAttnRows;
    const Q4 none{nullptr, nullptr};
    const int dt = (md.D + tc5::kTc5Rows - 1) / tc5::kTc5Rows;
    auto pm = [&](int m) -> const Tc5Pre& { return h.pre[(size_t)l * kPreMats + m]; };
    if (tc)
      launch_tc5_gemm<kTc5Qkv>(a, T, (md.QKV + tc5::kTc5Rows - 1) / tc5::kTc5Rows, md.QKV, md.D, L.qkv, none, L.qkv_b,
                               a.xh, a.xl, nullptr, nullptr, nullptr, pm(kPreQkv), st);
    else
      LWE_GEMM(lwe_gemm_qkv, kGemmRows, md.QKV, md.D, T, a, T, l, rope_epi ? 1 : 0);
    if (one_per_slot) {
      if (h.attn_split)
        launch_attention_split<true>(a, h, T, st);
      else
        launch_attention_t<true>(a, T, st);
    } else {
      if (!rope_epi) lwe_launch(lwe_rope_kv, dim3(T, md.NKV), dim3(64), 0, st, a, T);
      // a few tokens (a verify forward) over a long cache: split the positions across CTAs
      if (T <= kLweSplitAttnRows)
        launch_attention_split<false>(a, h, T, st);
      else
        launch_attention_t<false>(a, T, st);
    }
    // proj + residual; norm2 -> N2 (x3 buffer when folded, else a norm kernel into xh)
    LweArgs n2 = a;
    if (fold) {
      n2.xh = a.xh3;
      n2.xl = a.xl3;
      if (tc)
        launch_tc5_gemm<kTc5Resid>(a, T, dt, md.D, md.D, L.proj, none, L.proj_b, a.xh, a.xl, L.norm2, a.xh3, a.xl3,
                                   pm(kPreProj), st);
      else
        LWE_GEMM(lwe_gemm_resid, kGemmRows, md.D, md.D, T, a, T, L.proj, L.proj_b, md.D, L.norm2, a.xh3, a.xl3, a.ldx);
    } else {
      LWE_GEMM(lwe_gemm_resid, kGemmRows, md.D, md.D, T, a, T, L.proj, L.proj_b, md.D, nullptr, nullptr, nullptr, 0);
      lwe_launch(lwe_norm_split<false>, dim3(T), dim3(128), 0, st, a, T, L.norm2, (const int*)nullptr);
    }
    if (md.arch == 0) {
      // long forwards (prefill chunks): the persistent wide GEMM, activations read once per CTA
      if (tc)
        launch_tc5_gemm<kTc5W13>(a, T, (md.FF + 63) / 64, md.FF, md.D, L.w1, L.w3, nullptr, a.xh3, a.xl3, nullptr,
                                 nullptr, nullptr, pm(kPreW13), st);
      else if (!(T >= kW13WideRows && h.w13_wide && launch_w13_wide(n2, T, l, st)))
        LWE_GEMM(lwe_gemm_w13, 32, md.FF, md.D, T, n2, T, l);
    } else
      LWE_GEMM(lwe_gemm_fc, kGemmRows, md.FF, md.D, T, n2, T, l);
    LweArgs b = a;  // w2 / mlp.proj read the second activation buffer
    b.xh = a.xh2;
    b.xl = a.xl2;
    b.ldx = a.ldx2;
    // w2 + residual; the next layer's norm1 -> xh
    const float* ng = l + 1 < nl ? h.layers[l + 1].norm1 : nullptr;
    if (fold) {
      if (tc)
        launch_tc5_gemm<kTc5Resid>(a, T, dt, md.D, md.FF, L.w2, none, L.mproj_b, a.xh2, a.xl2, ng, a.xh, a.xl,
                                   pm(kPreW2), st);
      else
        LWE_GEMM(lwe_gemm_resid, kGemmRows, md.D, md.FF, T, b, T, L.w2, L.mproj_b, md.FF, ng, a.xh, a.xl, a.ldx);
    } else {
      LWE_GEMM(lwe_gemm_resid, kGemmRows, md.D, md.FF, T, b, T, L.w2, L.mproj_b, md.FF, nullptr, nullptr, nullptr, 0);
      if (ng) {
        lwe_launch(lwe_norm_split<false>, dim3(T), dim3(128), 0, st, a, T, ng, (const int*)nullptr);
      }
    }
  }
  if (lm_T > 0) {
    const int* src = lm_from_src ? a.lm_src : nullptr;
    int nblk = (md.vocab + kGemmRows - 1) / kGemmRows;
    if (logits == nullptr && lm_T >= kLmWideRows && h.lm_tc5 && g_lm_tc5_ok && !a.skip) {
      // many rows without logits (a batched decode step): the tcgen05 tile, one partial per vocab tile
      launch_lm_tc5(a, lm_T, md.norm_f, src, st, &nblk);
    } else {
      lwe_launch(lwe_norm_split<false>, dim3(lm_T), dim3(128), 0, st, a, lm_T, md.norm_f, src);
      // the same without tcgen05: the persistent wide GEMM, one partial per CTA
      if (!(logits == nullptr && lm_T >= kLmWideRows && h.lm_wide && launch_lm_wide(a, lm_T, st, &nblk)))
        LWE_GEMM_LM(md.vocab, lm_T, a, lm_T, logits);
    }
    lwe_launch(lwe_argmax_reduce, dim3((lm_T + 3) / 4), dim3(128), 0, st, a, lm_T, nblk);
  }
  return cudaGetLastError();
}

// ---- small bookkeeping kernels
__global__ void k_fill(const __grid_constant__ LweArgs a, const int32_t* ids, int n, int slot, int pos0, int lm_each) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    a.tok[i] = ids[i];
    a.slot[i] = slot;
    a.pos[i] = pos0 + i;
    if (lm_each) a.lm_src[i] = i;
  }
  if (!lm_each && blockIdx.x == 0 && threadIdx.x == 0) a.lm_src[0] = n - 1;
}
void lwe_fill(LweArgs a, const int32_t* ids, int n, int slot, int pos0, int lm_each, cudaStream_t st) {
  k_fill<<<(n + 255) / 256, 256, 0, st>>>(a, ids, n, slot, pos0, lm_each);
  ++g_lwe_launches;
}
void lwe_first(LweArgs a, int32_t* out_ids, int32_t* status, int eos, int forwards, int32_t* stream, cudaStream_t st) {
  lwe_first_token<<<1, 1, 0, st>>>(a.amax, out_ids, status, eos, forwards, stream);
  ++g_lwe_launches;
}
void lwe_mark_time(int32_t* status, int idx, cudaStream_t st) { lwe_mark<<<1, 1, 0, st>>>(status, idx); }

// Batched prefill: the host plan lists every prompt token of every sequence (its slot, position and
// index into the concatenated prompt ids); a forward takes tmax consecutive plan entries.
__global__ void k_gather(int32_t* tok, const int32_t* ids, const int32_t* src, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) tok[i] = ids[src[i]];
}
void lwe_gather(int32_t* tok, const int32_t* ids, const int32_t* src, int n, cudaStream_t st) {
  k_gather<<<(n + 255) / 256, 256, 0, st>>>(tok, ids, src, n);
  ++g_lwe_launches;
}
// First id of each sequence whose prompt ended in this forward: lm row j belongs to slot lm_slot[j]
// (engine/infer.js:611-623 per sequence); counts[s] = 1 while running, -1 once stopped.
__global__ void k_batch_first(const int32_t* amax, const int32_t* lm_slot, int nlm, int max_new, int eos, int kv_len,
                              int32_t* out_ids, int32_t* counts, const int32_t* lens) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= nlm) return;
  const int s = lm_slot[j], id = amax[j];
  out_ids[(size_t)s * max_new] = id;
  const bool stop = id == eos || max_new <= 1 || lens[s] + 1 >= kv_len;
  counts[s] = stop ? -1 : 1;
}
void lwe_batch_first(const int32_t* amax, const int32_t* lm_slot, int nlm, int max_new, int eos, int kv_len,
                     int32_t* out_ids, int32_t* counts, const int32_t* lens, cudaStream_t st) {
  k_batch_first<<<(nlm + 127) / 128, 128, 0, st>>>(amax, lm_slot, nlm, max_new, eos, kv_len, out_ids, counts, lens);
  ++g_lwe_launches;
}
// Decode rows: token t = slot t, its last id and position (engine/infer.js:627: the id fed at
// position prompt_len + generated - 1).
__global__ void k_batch_decode_setup(const __grid_constant__ LweArgs a, int n, const int32_t* out_ids,
                                     const int32_t* counts, const int32_t* lens, int max_new) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n) return;
  const int c = counts[t] < 0 ? -counts[t] : counts[t];
  a.tok[t] = out_ids[(size_t)t * max_new + c - 1];
  a.slot[t] = t;
  a.pos[t] = lens[t] + c - 1;
  a.lm_src[t] = t;
}
void lwe_batch_decode_setup(LweArgs a, int n, const int32_t* out_ids, const int32_t* counts, const int32_t* lens,
                            int max_new, cudaStream_t st) {
  k_batch_decode_setup<<<(n + 127) / 128, 128, 0, st>>>(a, n, out_ids, counts, lens, max_new);
  ++g_lwe_launches;
}
void lwe_batch_advance(LweArgs a, int n, int max_new, int eos, int32_t* out_ids, int32_t* counts, const int32_t* lens,
                       cudaStream_t st) {
  lwe_launch(lwe_decode_advance, dim3((n + 127) / 128), dim3(128), 0, st, a, n, max_new, eos, out_ids, counts, lens);
}

// Number of sequences still running -> *active.
__global__ void k_count_active(const int32_t* counts, int n, int32_t* active) {
  __shared__ int tot;
  if (threadIdx.x == 0) tot = 0;
  __syncthreads();
  int c = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) c += counts[i] > 0;
  if (c) atomicAdd(&tot, c);
  __syncthreads();
  if (threadIdx.x == 0) *active = tot;
}
void lwe_count_active(const int32_t* counts, int n, int32_t* active, cudaStream_t st) {
  k_count_active<<<1, 256, 0, st>>>(counts, n, active);
  ++g_lwe_launches;
}

// GPT-2 penalised argmax per decode row (engine/infer.js:252-287) over logits [T][V]; the history of
// row t is the ids its sequence generated so far, out_ids[t][0..counts[t]).  Ids that are banned (the
// 3-gram rule) or recent (the last 32) are marked in two shared-memory bitmaps; the rest take a plain
// f32 argmax, the marked ones are scored in f64 exactly like the reference, and the two results are
// merged (lowest index on equal values).
__global__ void __launch_bounds__(256) lwe_argmax_pen(const float* logits, int V, int T, const int32_t* out_ids,
                                                      const int32_t* counts, int max_new, int32_t* amax) {
  extern __shared__ uint32_t bits[];  // [2][nwords]: banned, recent; then the banned-id list [max_new]
  __shared__ int nban;
  __shared__ float wv[8];
  __shared__ int wi[8];
  __shared__ double dv[8];
  __shared__ int di[8];
  const int t = blockIdx.x;
  if (t >= T) return;
  const int nwords = (V + 31) >> 5;
  uint32_t* ban = bits;
  uint32_t* rec = bits + nwords;
  int* ban_list = reinterpret_cast<int*>(bits + 2 * nwords);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int32_t* hist = out_ids + (size_t)t * max_new;
  const int n_past = counts[t] < 0 ? -counts[t] : counts[t];
  for (int i = threadIdx.x; i < 2 * nwords; i += blockDim.x) bits[i] = 0u;
  if (threadIdx.x == 0) nban = 0;
  __syncthreads();
  const int rwin = max(0, n_past - 32);
  if (n_past >= 2) {
    const int t1 = hist[n_past - 2], t2 = hist[n_past - 1];
    for (int k = threadIdx.x; k < n_past - 2; k += blockDim.x)
      if (hist[k] == t1 && hist[k + 1] == t2) {
        const int id = hist[k + 2];
        const uint32_t old = atomicOr(&ban[id >> 5], 1u << (id & 31));
        if (!(old & (1u << (id & 31)))) {
          ban_list[atomicAdd(&nban, 1)] = id;  // distinct ids, fewer than n_past <= max_new
        }
      }
  }
  for (int k = rwin + threadIdx.x; k < n_past; k += blockDim.x) {
    const int id = hist[k];
    atomicOr(&rec[id >> 5], 1u << (id & 31));
  }
  __syncthreads();
  // plain argmax over unmarked ids
  const float* row = logits + (size_t)t * V;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const uint32_t m = (ban[i >> 5] | rec[i >> 5]) >> (i & 31);
    const float v = row[i];
    if (!(m & 1u) && v > best) {  // ids rise per thread: strict > keeps the lowest
      best = v;
      bidx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) {
      best = ov;
      bidx = oi;
    }
  }
  if (lane == 0) {
    wv[warp] = best;
    wi[warp] = bidx;
  }
  // marked ids: banned (from the list) and recent (from the history window), scored in f64
  double pb = -INFINITY;
  int pi = 0x7fffffff;
  const int nb = nban;
  for (int k = threadIdx.x; k < nb + (n_past - rwin); k += blockDim.x) {
    const int id = k < nb ? ban_list[k] : hist[rwin + k - nb];
    double v = row[id];
    if ((ban[id >> 5] >> (id & 31)) & 1u) v = -1e9;
    if (((rec[id >> 5] >> (id & 31)) & 1u) && v > -1e8) v = v > 0 ? v / 1.15 : v * 1.15;
    if (v > pb || (v == pb && id < pi)) {
      pb = v;
      pi = id;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double ov = __shfl_xor_sync(0xffffffffu, pb, o);
    const int oi = __shfl_xor_sync(0xffffffffu, pi, o);
    if (ov > pb || (ov == pb && oi < pi)) {
      pb = ov;
      pi = oi;
    }
  }
  if (lane == 0) {
    dv[warp] = pb;
    di[warp] = pi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      const double a = wv[w];
      if (a > bv || (a == bv && wi[w] < bi)) {
        bv = a;
        bi = wi[w];
      }
      if (dv[w] > bv || (dv[w] == bv && di[w] < bi)) {
        bv = dv[w];
        bi = di[w];
      }
    }
    amax[t] = bi;
  }
}
size_t lwe_argmax_pen_smem(int V, int max_new) { return (size_t)2 * ((V + 31) / 32) * 4 + (size_t)max_new * 4; }
void lwe_penalised_argmax(const float* logits, int V, int T, const int32_t* out_ids, const int32_t* counts, int max_new,
                          int32_t* amax, cudaStream_t st) {
  lwe_argmax_pen<<<T, 256, lwe_argmax_pen_smem(V, max_new), st>>>(logits, V, T, out_ids, counts, max_new, amax);
  ++g_lwe_launches;
}


// ---------------------------------------------------------------------------------------------
// Prompt-lookup speculation on the token-batch engine (engine/webgpu.js:1239-1270 with lookupDraft
// engine/webgpu.js:846-865): every iteration is one CUDA graph replay of prepare (draft lookup over
// the device-resident history, verify rows) -> forward over spec_k + 1 rows -> accept.  The loop
// state lives in device memory (SpecState words); once the loop is finished the replays are no-ops.
// ---------------------------------------------------------------------------------------------
enum SpecWord { SP_HLEN = 0, SP_GEN, SP_CACHE, SP_DONE, SP_HITS, SP_TRIES, SP_FWD, SP_TOK, SP_DL, SP_STOP, SP_POS0 };

// State after the prefill: history = prompt + first id (already in out_ids[0]).
__global__ void k_spec_init(int32_t* sp, const int32_t* ids, int n, const int32_t* out_ids, int max_new, int eos,
                            int kv_len, int prefill_forwards) {
  int32_t* hist = sp + kSpecHist;
  for (int i = threadIdx.x; i < n; i += blockDim.x) hist[i] = ids[i];
  if (threadIdx.x == 0) {
    const int tok = out_ids[0];
    hist[n] = tok;
    sp[SP_HLEN] = n + 1;
    sp[SP_GEN] = 1;
    sp[SP_CACHE] = n < kv_len - 1 ? n : kv_len - 1;
    sp[SP_TOK] = tok;
    sp[SP_HITS] = 0;
    sp[SP_TRIES] = 0;
    sp[SP_FWD] = prefill_forwards;
    sp[SP_STOP] = tok == eos ? 0 : 1;
    sp[SP_DONE] = tok == eos ? 1 : 0;
    sp[SP_DL] = 0;
  }
}

// Draft lookup and the verify rows: row 0 = the last id at position cache, rows 1..dl = the draft;
// rows dl+1..T-1 repeat row dl (same id, same position: identical K/V writes, logits unused).
__global__ void k_spec_prepare(const __grid_constant__ LweArgs a, int32_t* sp, int spec_k, int ngram, int max_new,
                               int T, int slot) {
  pdl_enter();
  __shared__ int best;
  __shared__ int sdone;
  const int32_t* hist = sp + kSpecHist;
  const int kv_len = a.m.kv_len;
  const int hlen = sp[SP_HLEN], gen = sp[SP_GEN], cache = sp[SP_CACHE];
  if (threadIdx.x == 0) {
    best = -1;
    int d = sp[SP_DONE];
    if (!d && (gen >= max_new || cache >= kv_len - 1)) d = 1;  // engine/webgpu.js:1239
    sdone = d;
    if (d) sp[SP_DONE] = 1;
  }
  __syncthreads();
  if (sdone) return;
  // latest earlier occurrence of the last `ngram` ids (engine/webgpu.js:846-865)
  if (hlen >= ngram + 1) {
    const int limit = hlen - ngram;
    int b = -1;
    for (int i = threadIdx.x; i < limit; i += blockDim.x) {
      bool ok = true;
      for (int j = 0; j < ngram; ++j)
        if (hist[i + j] != hist[hlen - ngram + j]) {
          ok = false;
          break;
        }
      if (ok) b = i;
    }
    if (b >= 0) atomicMax(&best, b);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const int i = best;
    int dl = 0;
    int32_t* draft = sp + kSpecDraft;
    if (i >= 0)
      for (int t = 0; t < spec_k && i + ngram + t < hlen; ++t) draft[dl++] = hist[i + ngram + t];
    if (cache + dl > kv_len - 1) dl = kv_len - 1 - cache;  // verify rows stay inside the cache
    sp[SP_DL] = dl;
    sp[SP_POS0] = cache;
    sp[SP_TRIES] += 1;
    for (int r = 0; r < T; ++r) {
      const int e = r < dl ? r : dl;
      a.tok[r] = e == 0 ? sp[SP_TOK] : draft[e - 1];
      a.pos[r] = cache + e;
      a.slot[r] = slot;
      a.lm_src[r] = r;
    }
  }
}

// engine/webgpu.js:1249-1268: accept r[0], then r[k+1] while r[k] == draft[k].
__global__ void k_spec_accept(const int32_t* amax, int32_t* sp, int32_t* out_ids, int max_new, int eos,
                              int32_t* stream) {
  pdl_enter();
  if (threadIdx.x != 0 || sp[SP_DONE]) return;
  int32_t* hist = sp + kSpecHist;
  const int32_t* draft = sp + kSpecDraft;
  const int dl = sp[SP_DL], pos0 = sp[SP_POS0];
  int gen = sp[SP_GEN], hlen = sp[SP_HLEN], hits = sp[SP_HITS];
  const int r0 = amax[0];
  stream_publish(stream, gen, r0, 1);
  out_ids[gen++] = r0;
  hist[hlen++] = r0;
  int cache = pos0 + 1, tok = r0;
  if (r0 != eos && dl > 0) {
    for (int k = 0; k < dl; ++k) {
      if (amax[k] != draft[k]) break;
      if (gen >= max_new) break;
      const int nxt = amax[k + 1];
      ++hits;
      stream_publish(stream, gen, nxt, 2);
      out_ids[gen++] = nxt;
      hist[hlen++] = nxt;
      cache = pos0 + 2 + k;
      tok = nxt;
      if (nxt == eos) break;
    }
  }
  sp[SP_GEN] = gen;
  sp[SP_HLEN] = hlen;
  sp[SP_HITS] = hits;
  sp[SP_CACHE] = cache;
  sp[SP_TOK] = tok;
  sp[SP_FWD] += 1;
  if (tok == eos) {
    sp[SP_STOP] = 0;
    sp[SP_DONE] = 1;
  }
}

// Status words of the generate call from the loop state.
__global__ void k_spec_finish(const int32_t* sp, int32_t* status) {
  status[ST_NGEN] = sp[SP_GEN];
  status[ST_STOP] = sp[SP_STOP];
  status[ST_HITS] = sp[SP_HITS];
  status[ST_TRIES] = sp[SP_TRIES];
  status[ST_FORWARDS] = sp[SP_FWD];
  const uint64_t t = globaltimer();
  status[ST_TEND] = (int32_t)(uint32_t)t;
  status[ST_TEND + 1] = (int32_t)(uint32_t)(t >> 32);
}

void lwe_spec_init(int32_t* sp, const int32_t* ids, int n, const int32_t* out_ids, int max_new, int eos, int kv_len,
                   int prefill_forwards, cudaStream_t st) {
  k_spec_init<<<1, 256, 0, st>>>(sp, ids, n, out_ids, max_new, eos, kv_len, prefill_forwards);
  ++g_lwe_launches;
}
cudaError_t lwe_spec_iteration(LweArgs a, const LweHost& h, int32_t* sp, int32_t* out_ids, int spec_k, int ngram,
                               int max_new, int eos, int slot, int32_t* stream, cudaStream_t st) {
  const int T = spec_k + 1;
  g_lwe_pdl = h.pdl != 0;
  lwe_launch(k_spec_prepare, dim3(1), dim3(256), 0, st, a, sp, spec_k, ngram, max_new, T, slot);
  LweArgs f = a;
  f.skip = sp + SP_DONE;
  const cudaError_t e = lwe_forward(f, h, T, T, false, nullptr, false, st);
  if (e != cudaSuccess) return e;
  lwe_launch(k_spec_accept, dim3(1), dim3(32), 0, st, (const int32_t*)a.amax, sp, out_ids, max_new, eos, stream);
  return cudaGetLastError();
}
void lwe_spec_finish(const int32_t* sp, int32_t* status, cudaStream_t st) {
  k_spec_finish<<<1, 1, 0, st>>>(sp, status);
  ++g_lwe_launches;
}

}  // namespace mllm
