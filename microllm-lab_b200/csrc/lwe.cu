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

#include "device_common.cuh"
#include "engine.cuh"
#include "lwe.cuh"
#include "q4mma.cuh"

namespace mllm {

constexpr int kLweTBW = 8;  // 64 tokens per GEMM CTA
constexpr int kLweBT = 8 * kLweTBW;

// ---------------------------------------------------------------------------------------------
__global__ void lwe_embed(const __grid_constant__ LweArgs a, int T) {
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
}

// RMSNorm / LayerNorm of X[src[i]] (or X[i]) -> fp16 hi/lo rows i of xh/xl.  One CTA per row.
__global__ void lwe_norm_split(const __grid_constant__ LweArgs a, int T, const float* g, const int* src) {
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
  __half* oh = a.xh + (size_t)i * a.ldx;
  __half* ol = a.xl + (size_t)i * a.ldx;
  if (md.arch == 0) {
    const float inv = 1.f / sqrtf(s2 / D + 1e-6f);  // engine/infer.js:134-143
    for (int k = threadIdx.x; k < D; k += blockDim.x) split_hi_lo(x[k] * inv * g[k], oh[k], ol[k]);
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
    for (int k = threadIdx.x; k < D; k += blockDim.x) split_hi_lo(fmaf((x[k] - mean) * inv, g[k], g[D + k]), oh[k], ol[k]);
  }
}

// QKV GEMM: qkv[t][r] = W_qkv[r] . norm1(x_t) (+ bias)
__global__ void __launch_bounds__(kGemmThreads) lwe_gemm_qkv(const __grid_constant__ LweArgs a, int T, int l) {
  extern __shared__ __align__(16) unsigned char smem[];
  const LayerDev& L = a.m.layers[l];
  const int R = a.m.QKV, K = a.m.D;
  const float* bias = L.qkv_b;
  float* out = a.qkv;
  q4_gemm_tile<kLweTBW>(reinterpret_cast<const uint8_t*>(L.qkv.w), L.qkv.s, a.xh, a.xl, a.ldx, R, K, T,
                        blockIdx.x * kGemmRows, blockIdx.y * kLweBT, smem,
                        [&](int r, int t, float v) { out[(size_t)t * R + r] = bias ? v + bias[r] : v; });
}

// RoPE on k (and on the q heads of the group) at each token's position, then the K/V cache write
// (engine/infer.js:436-464).  grid (T, NKV), 64 threads: thread d < 32 rotates pair (d, d + 32).
__global__ void lwe_rope_kv(const __grid_constant__ LweArgs a, int T) {
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

// Attention of the `rep` query heads of kv head g for token t over positions 0..pos[t] of its slot
// (engine/infer.js:466-495), online softmax, 4 lanes per position (16 dims each), 4 warps.
// Output rows are written as fp16 hi/lo into xh/xl for the proj GEMM.
__global__ void __launch_bounds__(128) lwe_attention(const __grid_constant__ LweArgs a, int T) {
  const int t = blockIdx.x, g = blockIdx.y;
  if (t >= T) return;
  const ModelDev& md = a.m;
  const int NKV = md.NKV, rep = md.NH / NKV, pos = a.pos[t], npos = pos + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, qd = lane & 3, pg = lane >> 2;
  __shared__ float part[4][kLweMaxRep][68];
  const float* qrow = a.qkv + (size_t)t * md.QKV + g * rep * 64;
  float q[kLweMaxRep][16];
#pragma unroll
  for (int h = 0; h < kLweMaxRep; ++h)
#pragma unroll
    for (int i = 0; i < 16; ++i) q[h][i] = h < rep ? qrow[h * 64 + qd * 16 + i] : 0.f;
  const size_t base = ((size_t)a.layer * NKV + g) * md.kv_len;
  const float* kc = a.kc[a.slot[t]] + base * 64;
  const float* vc = a.vc[a.slot[t]] + base * 64;
  float m[kLweMaxRep], lsum[kLweMaxRep], o[kLweMaxRep][16];
#pragma unroll
  for (int h = 0; h < kLweMaxRep; ++h) {
    m[h] = -INFINITY;
    lsum[h] = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) o[h][i] = 0.f;
  }
  for (int p0 = warp * 8; p0 < npos; p0 += 32) {
    const int p = p0 + pg;
    const bool valid = p < npos;
    float4 kk[4], vv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kk[j] = valid ? ldcg_f4(kc + (size_t)p * 64 + qd * 16 + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
      vv[j] = valid ? ldcg_f4(vc + (size_t)p * 64 + qd * 16 + 4 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int h = 0; h < kLweMaxRep; ++h) {
      if (h >= rep) break;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s = fmaf(q[h][4 * j], kk[j].x, s);
        s = fmaf(q[h][4 * j + 1], kk[j].y, s);
        s = fmaf(q[h][4 * j + 2], kk[j].z, s);
        s = fmaf(q[h][4 * j + 3], kk[j].w, s);
      }
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      const float sc = valid ? s * 0.125f : -INFINITY;  // 1/sqrt(64), exact (engine/infer.js:466)
      const float newm = fmaxf(m[h], warp_max(sc));
      const float e = valid ? expf(sc - newm) : 0.f;
      const float corr = m[h] == -INFINITY ? 0.f : expf(m[h] - newm);
      lsum[h] = fmaf(lsum[h], corr, warp_sum(qd == 0 ? e : 0.f));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[h][4 * j] = fmaf(e, vv[j].x, o[h][4 * j] * corr);
        o[h][4 * j + 1] = fmaf(e, vv[j].y, o[h][4 * j + 1] * corr);
        o[h][4 * j + 2] = fmaf(e, vv[j].z, o[h][4 * j + 2] * corr);
        o[h][4 * j + 3] = fmaf(e, vv[j].w, o[h][4 * j + 3] * corr);
      }
      m[h] = newm;
    }
  }
#pragma unroll
  for (int h = 0; h < kLweMaxRep; ++h) {
    if (h >= rep) break;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[h][i] += __shfl_xor_sync(0xffffffffu, o[h][i], 4);
      o[h][i] += __shfl_xor_sync(0xffffffffu, o[h][i], 8);
      o[h][i] += __shfl_xor_sync(0xffffffffu, o[h][i], 16);
    }
    if (lane == 0) {
      part[warp][h][0] = m[h];
      part[warp][h][1] = lsum[h];
    }
    if (pg == 0)
#pragma unroll
      for (int i = 0; i < 16; ++i) part[warp][h][4 + qd * 16 + i] = o[h][i];
  }
  __syncthreads();
  // combine the 4 warps: thread (h, d) for h < rep, d < 64 -> 128 threads cover 2 heads per pass
  for (int hd = threadIdx.x; hd < rep * 64; hd += blockDim.x) {
    const int h = hd >> 6, d = hd & 63;
    float M = -INFINITY;
    for (int w = 0; w < 4; ++w) M = fmaxf(M, part[w][h][0]);
    float Ls = 0.f, r = 0.f;
    for (int w = 0; w < 4; ++w) {
      if (part[w][h][1] > 0.f) {
        const float f = expf(part[w][h][0] - M);
        Ls = fmaf(part[w][h][1], f, Ls);
        r = fmaf(part[w][h][4 + d], f, r);
      }
    }
    const size_t off = (size_t)t * a.ldx + (g * rep + h) * 64 + d;
    split_hi_lo(r / Ls, a.xh[off], a.xl[off]);
  }
}

// GEMM with a residual epilogue: x[t][r] += W[r] . in_t (+ bias)  (proj and w2)
__global__ void __launch_bounds__(kGemmThreads) lwe_gemm_resid(const __grid_constant__ LweArgs a, int T, Q4 w,
                                                               const float* bias, int K) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int R = a.m.D;
  float* x = a.x;
  q4_gemm_tile<kLweTBW>(reinterpret_cast<const uint8_t*>(w.w), w.s, a.xh, a.xl, a.ldx, R, K, T,
                        blockIdx.x * kGemmRows, blockIdx.y * kLweBT, smem, [&](int r, int t, float v) {
                          x[(size_t)t * R + r] += bias ? v + bias[r] : v;
                        });
}

// w1/w3 paired GEMM with the SiLU*mul epilogue (engine/infer.js:178-183, 522-524); output written as
// fp16 hi/lo into the second activation buffer (xh2/xl2).  32 matrix rows per CTA.
__global__ void __launch_bounds__(kGemmThreads) lwe_gemm_w13(const __grid_constant__ LweArgs a, int T, int l) {
  extern __shared__ __align__(16) unsigned char smem[];
  const LayerDev& L = a.m.layers[l];
  const int FF = a.m.FF, K = a.m.D;
  const RowsPaired rows{reinterpret_cast<const uint8_t*>(L.w1.w), L.w1.s, reinterpret_cast<const uint8_t*>(L.w3.w),
                        L.w3.s, FF, (int)blockIdx.x * 32, K >> 1, K >> 5};
  float acc[kLweTBW][4];
  const int t0 = blockIdx.y * kLweBT;
  q4_gemm_core<kLweTBW>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int ia = warp * 16 + gid;  // A row (w1); the B row (w3) of the same matrix row is ia + 8
  if (!rows.valid(ia)) return;
  const int r = rows.mrow(ia);
#pragma unroll
  for (int b = 0; b < kLweTBW; ++b) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int tok = t0 + b * 8 + 2 * t + e;
      if (tok >= T) continue;
      const float u = acc[b][e], v = acc[b][2 + e];
      const size_t off = (size_t)tok * a.ldx2 + r;
      split_hi_lo((u / (1.f + expf(-u))) * v, a.xh2[off], a.xl2[off]);
    }
  }
}

// GPT-2 fc GEMM with bias + GELU (engine/infer.js:512-515, 166-171) -> fp16 hi/lo (xh2/xl2)
__global__ void __launch_bounds__(kGemmThreads) lwe_gemm_fc(const __grid_constant__ LweArgs a, int T, int l) {
  extern __shared__ __align__(16) unsigned char smem[];
  const LayerDev& L = a.m.layers[l];
  const int FF = a.m.FF, K = a.m.D;
  const float* bias = L.fc_b;
  q4_gemm_tile<kLweTBW>(reinterpret_cast<const uint8_t*>(L.w1.w), L.w1.s, a.xh, a.xl, a.ldx, FF, K, T,
                        blockIdx.x * kGemmRows, blockIdx.y * kLweBT, smem, [&](int r, int t, float v) {
                          if (bias) v += bias[r];
                          const float gl = 0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
                          split_hi_lo(gl, a.xh2[(size_t)t * a.ldx2 + r], a.xl2[(size_t)t * a.ldx2 + r]);
                        });
}

// lm_head GEMM over the T rows in xh/xl with a per-CTA argmax epilogue: for each token, the best
// (value, lowest index) over the CTA's 64 vocab rows goes to pval/pidx[blockIdx.x][t].  Optional
// logits store [t][V].
__global__ void __launch_bounds__(kGemmThreads) lwe_gemm_lm(const __grid_constant__ LweArgs a, int T, float* logits) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int V = a.m.vocab, K = a.m.D;
  const int r0 = blockIdx.x * kGemmRows, t0 = blockIdx.y * kLweBT;
  float acc[kLweTBW][4];
  const RowsLinear rows{reinterpret_cast<const uint8_t*>(a.m.lm.w), a.m.lm.s, V, r0, K >> 1, K >> 5};
  q4_gemm_core<kLweTBW>(rows, a.xh, a.xl, a.ldx, K, T, t0, smem, acc);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, gid = lane >> 2, t = lane & 3;
  const int ra = r0 + warp * 16 + gid, rb = ra + 8;
  __syncthreads();  // the pipeline buffers are reused below
  float* bv = reinterpret_cast<float*>(smem);            // [4 warps][kLweBT]
  int* bi = reinterpret_cast<int*>(bv + 4 * kLweBT);     // [4 warps][kLweBT]
#pragma unroll
  for (int b = 0; b < kLweTBW; ++b) {
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

// One greedy step of the replicated multi-sequence decode for every active slot: record the new id,
// apply the stop rules of engine/infer.js:617-639 and advance token and position.
__global__ void lwe_decode_advance(const __grid_constant__ LweArgs a, int T, int max_new, int eos,
                                   int32_t* out_ids, int32_t* counts, const int32_t* prompt_len) {
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
__global__ void lwe_first_token(const int32_t* amax, int32_t* out_ids, int32_t* status, int eos, int forwards) {
  const int id = amax[0];
  out_ids[0] = id;
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
size_t lwe_gemm_smem() { return q4_gemm_smem_bytes<kLweTBW>(); }

static inline dim3 gemm_grid(int rows_per_cta, int R, int T) {
  return dim3((R + rows_per_cta - 1) / rows_per_cta, (T + kLweBT - 1) / kLweBT);
}

// A forward over T tokens whose ids/slots/positions are already in a.tok/a.slot/a.pos.  When
// lm_T > 0 the lm_head runs on lm_T rows — the token rows a.lm_src[0..lm_T) when lm_from_src, else
// rows 0..lm_T — and leaves the argmax per row in a.amax; logits (nullable) receives [lm_T][V].
cudaError_t lwe_forward(LweArgs a, const LweHost& h, int T, int lm_T, bool lm_from_src, float* logits,
                        cudaStream_t st) {
  const ModelDev& md = a.m;
  const size_t sm = lwe_gemm_smem();
  lwe_embed<<<T, 128, 0, st>>>(a, T);
  for (int l = 0; l < md.n_layers; ++l) {
    const LayerDev& L = h.layers[l];
    a.layer = l;
    lwe_norm_split<<<T, 128, 0, st>>>(a, T, L.norm1, nullptr);
    lwe_gemm_qkv<<<gemm_grid(kGemmRows, md.QKV, T), kGemmThreads, sm, st>>>(a, T, l);
    lwe_rope_kv<<<dim3(T, md.NKV), 64, 0, st>>>(a, T);
    lwe_attention<<<dim3(T, md.NKV), 128, 0, st>>>(a, T);
    lwe_gemm_resid<<<gemm_grid(kGemmRows, md.D, T), kGemmThreads, sm, st>>>(a, T, L.proj, L.proj_b, md.D);
    lwe_norm_split<<<T, 128, 0, st>>>(a, T, L.norm2, nullptr);
    if (md.arch == 0)
      lwe_gemm_w13<<<gemm_grid(32, md.FF, T), kGemmThreads, sm, st>>>(a, T, l);
    else
      lwe_gemm_fc<<<gemm_grid(kGemmRows, md.FF, T), kGemmThreads, sm, st>>>(a, T, l);
    LweArgs b = a;  // w2 / mlp.proj read the second activation buffer
    b.xh = a.xh2;
    b.xl = a.xl2;
    b.ldx = a.ldx2;
    lwe_gemm_resid<<<gemm_grid(kGemmRows, md.D, T), kGemmThreads, sm, st>>>(b, T, L.w2, L.mproj_b, md.FF);
  }
  if (lm_T > 0) {
    lwe_norm_split<<<lm_T, 128, 0, st>>>(a, lm_T, md.norm_f, lm_from_src ? a.lm_src : nullptr);
    const dim3 g = gemm_grid(kGemmRows, md.vocab, lm_T);
    lwe_gemm_lm<<<g, kGemmThreads, sm, st>>>(a, lm_T, logits);
    lwe_argmax_reduce<<<(lm_T + 3) / 4, 128, 0, st>>>(a, lm_T, (int)g.x);
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
}
void lwe_first(LweArgs a, int32_t* out_ids, int32_t* status, int eos, int forwards, cudaStream_t st) {
  lwe_first_token<<<1, 1, 0, st>>>(a.amax, out_ids, status, eos, forwards);
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
}
void lwe_batch_advance(LweArgs a, int n, int max_new, int eos, int32_t* out_ids, int32_t* counts, const int32_t* lens,
                       cudaStream_t st) {
  lwe_decode_advance<<<(n + 127) / 128, 128, 0, st>>>(a, n, max_new, eos, out_ids, counts, lens);
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
}

}  // namespace mllm
