// Single-token persistent decode kernel: the greedy decode loop of engine/infer.js:625-639 (and the
// GPT-2 penalised argmax of engine/infer.js:252-287), one cooperative launch, one CTA per SM.
//
// Same protocol as the general kernel in decode.cu (flag-in-data exchange words, one buffer per
// layer and stage, an all-CTA argmax exchange that closes each forward), written for a small
// register footprint: little state lives across stages, the large stages are separate functions,
// and weight rows are requested before the wait that precedes their use.
//
// Per layer: QKV rows (warp per row) -> attention (one CTA per head) -> proj rows + residual ->
// w1/w3 rows + SiLU*mul (GPT-2: fc + bias + GELU) -> w2 rows + residual.
#include <cuda_runtime.h>

#include "device_common.cuh"
#include "engine.cuh"

namespace mllm {
namespace d1 {

// Shared-memory layout (4-byte words) for one token row.
struct Lay {
  float* xs;     // [D] residual stream
  float* act;    // [actw] stage input / normalised row / scratch
  float* wpart;  // [kWarps][68] attention partials
  float* red;    // [2][kWarps] norm partial sums
  int* hist;     // [kv_len + 64] prompt + generated ids
  int* pen;      // [kv_len + 128] GPT-2 banned / recent ids
  int* misc;     // [32]
  double* cval;  // [kWarps]
  int* cidx;     // [kWarps]
  uint32_t* lmw; // [lm_rpc][D/8] resident lm_head words (when RunArgs::lm_rpc > 0)
  float* lms;    // [lm_rpc][D/32] their scales
};

__device__ __forceinline__ int act_width(const ModelDev& md, int grid) {
  int w = max(max(md.D, md.QKV), md.FF);
  w = max(w, 3 * grid + 4);
  return (w + 3) & ~3;
}

__device__ __forceinline__ Lay layout(const ModelDev& md, float* smem) {
  Lay L;
  float* p = smem;
  L.xs = p; p += md.D;
  L.act = p; p += act_width(md, gridDim.x);
  L.wpart = p; p += kWarps * 68;
  L.red = p; p += 2 * kWarps;
  L.hist = reinterpret_cast<int*>(p); p += md.kv_len + 64;
  L.pen = reinterpret_cast<int*>(p); p += md.kv_len + 128;
  L.misc = reinterpret_cast<int*>(p); p += 32;
  p = reinterpret_cast<float*>(((uintptr_t)p + 7) & ~(uintptr_t)7);
  L.cval = reinterpret_cast<double*>(p); p += 2 * kWarps;
  L.cidx = reinterpret_cast<int*>(p); p += kWarps;
  p = reinterpret_cast<float*>(((uintptr_t)p + 15) & ~(uintptr_t)15);
  L.lmw = reinterpret_cast<uint32_t*>(p);
  L.lms = nullptr;
  return L;
}

// lm_head rows resident in shared memory: words then scales, both 16-byte aligned.
__device__ __forceinline__ void lm_resident_ptrs(const ModelDev& md, int rpc, Lay& L) {
  const size_t wwords = ((size_t)rpc * (md.D >> 3) + 3) & ~(size_t)3;
  L.lms = reinterpret_cast<float*>(L.lmw + wwords);
}


// Wait for the n contiguous words src[0..n) (tag == tag) and store their values to dst[0..n).
// Every thread of the CTA calls it; returns false (everywhere) when the wait gave up.
__device__ __noinline__ bool poll_vec(const uint64_t* src, float* dst, int n, uint32_t tag, int* err, uint64_t limit,
                                      int sleep_ns = 0) {
  bool ok = true;
  const uint64_t t0 = globaltimer();
  for (int base = threadIdx.x; base < n && ok; base += 8 * kThreads) {
    uint32_t pending = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (base + k * kThreads < n) pending |= 1u << k;
    int rounds = 0;
    while (pending) {
      uint64_t v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (pending & (1u << k)) v[k] = ll_load(src + base + k * kThreads);
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if ((pending & (1u << k)) && (uint32_t)(v[k] >> 32) == tag) {
          dst[base + k * kThreads] = __uint_as_float((uint32_t)v[k]);
          pending &= ~(1u << k);
        }
      if (pending && sleep_ns) __nanosleep(sleep_ns);
      if (pending && ((++rounds & 31) == 0)) {
        if (*(volatile int*)err || globaltimer() - t0 > limit) {
          atomicCAS(err, 0, 1);
          ok = false;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok);
}

// Wait for the residual row src[0..D) (D <= 4 * kThreads) and store it to xs; for RMSNorm also
// store x * gain to act and leave each warp's sum of squares in red[warp], so that 1 / RMS is
// available to every warp after the call without another pass (engine/infer.js:134-143 with the
// 1 / RMS factor applied to the dot products).  Returns false (everywhere) when the wait gave up.
__device__ __noinline__ bool poll_x_rms(const uint64_t* src, float* xs, float* act, float* red, int D, float g0, float g1,
                                        float g2, float g3, uint32_t tag, int* err, uint64_t limit, int sleep_ns) {
  const float g[4] = {g0, g1, g2, g3};
  uint32_t pending = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if ((int)threadIdx.x + kThreads * j < D) pending |= 1u << j;
  bool ok = true;
  float s2 = 0.f;
  const uint64_t t0 = globaltimer();
  int rounds = 0;
  while (pending) {
    uint64_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (pending & (1u << j)) v[j] = ll_load(src + threadIdx.x + kThreads * j);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if ((pending & (1u << j)) && (uint32_t)(v[j] >> 32) == tag) {
        const float x = __uint_as_float((uint32_t)v[j]);
        const int k = threadIdx.x + kThreads * j;
        xs[k] = x;
        act[k] = x * g[j];
        s2 = fmaf(x, x, s2);
        pending &= ~(1u << j);
      }
    if (pending && sleep_ns) __nanosleep(sleep_ns);
    if (pending && ((++rounds & 31) == 0)) {
      if (*(volatile int*)err || globaltimer() - t0 > limit) {
        atomicCAS(err, 0, 1);
        ok = false;
        break;
      }
    }
  }
  s2 = warp_sum(s2);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s2;
  return __syncthreads_and(ok);
}

__device__ __forceinline__ float rms_inv(const float* red, int D) {
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += red[w];
  return 1.f / sqrtf(s / D + 1e-6f);
}

// RMSNorm (engine/infer.js:134-143, eps 1e-6) or LayerNorm (engine/infer.js:147-164, eps 1e-5) of
// x[0..D) into out, with the gains (and biases) already in registers; fp32 statistics.
__device__ __noinline__ void norm_row(const float* x, float* out, float* red, int D, bool ln, float g0, float g1, float g2,
                                      float g3, float b0, float b1, float b2, float b3) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float g[4] = {g0, g1, g2, g3}, b[4] = {b0, b1, b2, b3};
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = threadIdx.x + kThreads * j;
    if (k < D) {
      s1 += x[k];
      s2 = fmaf(x[k], x[k], s2);
    }
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) {
    red[warp] = s1;
    red[kWarps + warp] = s2;
  }
  __syncthreads();
  s1 = 0.f;
  s2 = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    s1 += red[w];
    s2 += red[kWarps + w];
  }
  if (!ln) {
    const float inv = 1.f / sqrtf(s2 / D + 1e-6f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = threadIdx.x + kThreads * j;
      if (k < D) out[k] = x[k] * inv * g[j];
    }
  } else {
    const float mean = s1 / D;
    const float inv = 1.f / sqrtf(fmaxf(s2 / D - mean * mean, 0.f) + 1e-5f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = threadIdx.x + kThreads * j;
      if (k < D) out[k] = fmaf((x[k] - mean) * inv, g[j], b[j]);
    }
  }
  __syncthreads();
}

// One Q4 row's words for this lane: words lane + 32 j of the row (u32 = 8 elements).
template <int NWJ>
struct Row {
  uint32_t w[NWJ];
  float s[NWJ];
  __device__ __forceinline__ void load(const Q4& q, int row, int nwords, int lane) {
    const uint32_t* wr = q.w + (size_t)row * nwords;
    const float* sr = q.s + (size_t)row * (nwords >> 2);
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      w[j] = k < nwords ? ldv_u32(wr + k) : 0x88888888u;
      s[j] = k < nwords ? ldv_f32(sr + (k >> 2)) : 0.f;
    }
  }
  __device__ __forceinline__ float partial(const float* x, int nwords, int lane) const {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      if (k < nwords) acc = fmaf(word_dot(w[j], x + 8 * k), s[j], acc);
    }
    return acc;
  }
  __device__ __forceinline__ float dot(const float* x, int nwords, int lane) const {
    return warp_sum(partial(x, nwords, lane));
  }
  // Same with this lane's activations already in registers (xr[j] = x[8k..8k+7], k = lane + 32 j).
  __device__ __forceinline__ float dot_reg(const float (&xr)[NWJ][8], int nwords, int lane) const {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      if (k < nwords) {
        const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
        float t = nib_at(lo, 0) * xr[j][0];
        t = fmaf(nib_at(hi, 0), xr[j][1], t);
        t = fmaf(nib_at(lo, 1), xr[j][2], t);
        t = fmaf(nib_at(hi, 1), xr[j][3], t);
        t = fmaf(nib_at(lo, 2), xr[j][4], t);
        t = fmaf(nib_at(hi, 2), xr[j][5], t);
        t = fmaf(nib_at(lo, 3), xr[j][6], t);
        t = fmaf(nib_at(hi, 3), xr[j][7], t);
        acc = fmaf(t, s[j], acc);
      }
    }
    return warp_sum(acc);
  }
};

__device__ __forceinline__ void load_gains(const float* g, int D, bool ln, float (&gv)[4], float (&bv)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = threadIdx.x + kThreads * j;
    gv[j] = k < D ? ldv_f32(g + k) : 0.f;
    bv[j] = (ln && k < D) ? ldv_f32(g + D + k) : 0.f;
  }
}


// Causal attention of head h for the token at `pos` (engine/infer.js:422-495), split over `ns` CTAs
// by position: split sp covers positions [sp * P, (sp + 1) * P) of 0..pos, P = ceil((pos + 1) / ns).
// RoPE on q and on the new k, cache write by the last split of the group's first head, then online
// softmax over the split's positions with 4 lanes per position (16 dims each).  With one split the CTA
// publishes the head's 64 outputs; otherwise every split but the first publishes its partial
// (max, sum, 64 unnormalised outputs) to the partials area after the candidate words, and the first split
// merges them and publishes.
// SPLIT = false compiles the single-split form only (contexts of at most two rounds of positions).
template <bool SPLIT>
__device__ __noinline__ bool attention(const RunArgs& a, const Lay& S, int l, int unit, int pos, uint32_t tag) {
  const int h = SPLIT ? unit & 0xFF : unit;  // head, split, splits
  const int sp = SPLIT ? (unit >> 8) & 0xFF : 0, ns = SPLIT ? unit >> 16 : 1;
  const ModelDev& md = a.m;
  const ExchangeDev& x = a.x;
  const int D = md.D, NKV = md.NKV, rep = md.NH / md.NKV, kvh = h / rep;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* q = S.act;       // [64]
  float* kl = q + 64;     // [64]  new k
  float* vl = kl + 64;    // [64]  new v
  const bool rope = md.arch == 0 && md.rope_dim > 0;
  const int half = rope ? md.rope_dim / 2 : 1;
  // RoPE table values of this thread's pair (threads 0..31: q, 32..63: k), fetched before the wait.
  float c0 = 0.f, c1 = 0.f, s0 = 0.f, s1 = 0.f;
  if (rope && threadIdx.x < 2 * half) {
    const int d = threadIdx.x % half;
    const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
    const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
    c0 = ldv_f32(cs + d);
    c1 = ldv_f32(cs + d + half);
    s0 = ldv_f32(sn + d);
    s1 = ldv_f32(sn + d + half);
  }
  const uint64_t* qkv_l = x.qkv + (size_t)l * a.mmax * x.s_qkv;
  // q (64 words), k and v of the kv head (64 each): three contiguous runs
  bool ok = true;
  {
    const uint64_t t0 = globaltimer();
    const int i = threadIdx.x;  // 192 words, one per thread
    if (i < 192) {
      const uint64_t* src = i < 64 ? qkv_l + h * 64 + i
                            : i < 128 ? qkv_l + D + kvh * 64 + (i - 64)
                                      : qkv_l + D + NKV * 64 + kvh * 64 + (i - 128);
      int rounds = 0;
      for (;;) {
        const uint64_t v = ll_load(src);
        if ((uint32_t)(v >> 32) == tag) {
          q[i] = __uint_as_float((uint32_t)v);
          break;
        }
        if (((++rounds & 31) == 0) && (*(volatile int*)a.err || globaltimer() - t0 > (a.wait_ns ? a.wait_ns : kWaitNs))) {
          atomicCAS(a.err, 0, 1);
          ok = false;
          break;
        }
      }
    }
    if (!__syncthreads_and(ok)) return false;
  }
  if (rope && threadIdx.x < 2 * half) {
    float* v = threadIdx.x < half ? q : kl;
    const int d = threadIdx.x % half;
    const float a0 = v[d], a1 = v[d + half];
    v[d] = fmaf(-a1, s0, a0 * c0);
    v[d + half] = fmaf(a0, s1, a1 * c1);
  }
  __syncthreads();
  const size_t kv_base = ((size_t)l * NKV + kvh) * md.kv_len;
  if (h % rep == 0 && sp == ns - 1 && threadIdx.x < 128) {  // engine/infer.js:457-464
    const int d = threadIdx.x & 63;
    if (threadIdx.x < 64) a.kc[(kv_base + pos) * 64 + d] = kl[d];
    else a.vc[(kv_base + pos) * 64 + d] = vl[d];
  }
  const int qd = lane & 3, pg = lane >> 2;
  const int span = (pos + ns) / ns;  // ceil((pos + 1) / ns)
  const int p_lo = sp * span, p_hi = min(pos + 1, p_lo + span);
  float mrun = -INFINITY, lrun = 0.f, o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = 0.f;
  // Each round covers two 8-position slots per warp (positions r0 + pg and r0 + 64 + pg); the K and
  // V rows of both are requested together, then one online-softmax update.  The new position's k/v
  // come from shared memory.
  auto fetch = [&](int p, float4 (&kk)[4], float4 (&vv)[4]) {
    if (p < pos) {
      const float* kr = a.kc + (kv_base + p) * 64 + qd * 16;
      const float* vr = a.vc + (kv_base + p) * 64 + qd * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kk[j] = ldcg_f4(kr + 4 * j);
        vv[j] = ldcg_f4(vr + 4 * j);
      }
    } else if (p == pos) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kk[j] = *reinterpret_cast<const float4*>(kl + qd * 16 + 4 * j);
        vv[j] = *reinterpret_cast<const float4*>(vl + qd * 16 + 4 * j);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) kk[j] = vv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto score = [&](const float4 (&kk)[4], bool valid) {
    float part = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 qq = *reinterpret_cast<const float4*>(q + qd * 16 + 4 * j);
      part = fmaf(qq.x, kk[j].x, part);
      part = fmaf(qq.y, kk[j].y, part);
      part = fmaf(qq.z, kk[j].z, part);
      part = fmaf(qq.w, kk[j].w, part);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    return valid ? part * 0.125f : -INFINITY;  // 1/sqrt(64), exact (engine/infer.js:466)
  };
  for (int r0 = p_lo + warp * 8; r0 < p_hi; r0 += 2 * kWarps * 8) {
    const int pA = r0 + pg, pB = r0 + kWarps * 8 + pg;
    float4 kA[4], vA[4], kB[4], vB[4];
    fetch(pA, kA, vA);
    fetch(pB, kB, vB);
    const float sA = score(kA, pA < p_hi), sB = score(kB, pB < p_hi);
    const float newm = fmaxf(mrun, warp_max(fmaxf(sA, sB)));
    const float eA = pA < p_hi ? expf(sA - newm) : 0.f;
    const float eB = pB < p_hi ? expf(sB - newm) : 0.f;
    const float corr = mrun == -INFINITY ? 0.f : expf(mrun - newm);
    lrun = fmaf(lrun, corr, warp_sum(qd == 0 ? eA + eB : 0.f));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[4 * j] = fmaf(eB, vB[j].x, fmaf(eA, vA[j].x, o[4 * j] * corr));
      o[4 * j + 1] = fmaf(eB, vB[j].y, fmaf(eA, vA[j].y, o[4 * j + 1] * corr));
      o[4 * j + 2] = fmaf(eB, vB[j].z, fmaf(eA, vA[j].z, o[4 * j + 2] * corr));
      o[4 * j + 3] = fmaf(eB, vB[j].w, fmaf(eA, vA[j].w, o[4 * j + 3] * corr));
    }
    mrun = newm;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    o[i] += __shfl_xor_sync(0xffffffffu, o[i], 4);
    o[i] += __shfl_xor_sync(0xffffffffu, o[i], 8);
    o[i] += __shfl_xor_sync(0xffffffffu, o[i], 16);
  }
  float* wp = S.wpart + warp * 68;
  if (lane == 0) {
    wp[0] = mrun;
    wp[1] = lrun;
  }
  if (pg == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) wp[4 + qd * 16 + i] = o[i];
  }
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, S.wpart[w * 68]);
    float Ls = 0.f, r0 = 0.f, r1 = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float* pw = S.wpart + w * 68;
      if (pw[1] > 0.f) {
        const float f = expf(pw[0] - M);
        Ls = fmaf(pw[1], f, Ls);
        r0 = fmaf(pw[4 + 2 * lane], f, r0);
        r1 = fmaf(pw[4 + 2 * lane + 1], f, r1);
      }
    }
    if (ns == 1) {
      const float inv = 1.f / Ls;
      uint64_t* dst = x.att + (size_t)l * a.mmax * x.s_d + h * 64;
      ll_store(dst + 2 * lane, tag, r0 * inv);
      ll_store(dst + 2 * lane + 1, tag, r1 * inv);
    } else if (sp > 0) {
      // partial of this split: words 0 max, 1 sum, 2-3 zero, 4 + d unnormalised output d
      uint64_t* dst = x.cand + attn_partials_offset(gridDim.x, a.mmax) + (((size_t)l * md.NH + h) * kAttnSplits + sp) * kAttnPartWords;
      if (lane == 0) {
        ll_store(dst, tag, M);
        ll_store(dst + 1, tag, Ls);
        ll_store(dst + 2, tag, 0.f);
        ll_store(dst + 3, tag, 0.f);
      }
      ll_store(dst + 4 + 2 * lane, tag, r0);
      ll_store(dst + 5 + 2 * lane, tag, r1);
    } else {
      S.wpart[0] = M;  // lane-uniform values; lanes keep r0, r1
      S.wpart[1] = Ls;
      S.wpart[4 + 2 * lane] = r0;
      S.wpart[5 + 2 * lane] = r1;
    }
  }
  if (ns > 1 && sp == 0) {
    // first split: wait for the other splits' partials, merge, publish the head's outputs
    __syncthreads();
    float* part = S.act + 256;
    const uint64_t* src = x.cand + attn_partials_offset(gridDim.x, a.mmax) +
                          (((size_t)l * md.NH + h) * kAttnSplits + 1) * kAttnPartWords;
    if (!poll_vec(src, part, (ns - 1) * kAttnPartWords, tag, a.err, a.wait_ns ? a.wait_ns : kWaitNs,
                  a.poll_sleep_ns))
      return false;
    if (warp == 0) {
      float M = S.wpart[0];
      for (int q = 0; q < ns - 1; ++q)
        if (part[q * kAttnPartWords + 1] > 0.f) M = fmaxf(M, part[q * kAttnPartWords]);
      const float f0 = expf(S.wpart[0] - M);
      float Ls = S.wpart[1] * f0, r0 = S.wpart[4 + 2 * lane] * f0, r1 = S.wpart[5 + 2 * lane] * f0;
      for (int q = 0; q < ns - 1; ++q) {
        const float* pq = part + q * kAttnPartWords;
        if (pq[1] > 0.f) {
          const float f = expf(pq[0] - M);
          Ls = fmaf(pq[1], f, Ls);
          r0 = fmaf(pq[4 + 2 * lane], f, r0);
          r1 = fmaf(pq[5 + 2 * lane], f, r1);
        }
      }
      const float inv = 1.f / Ls;
      uint64_t* dst = x.att + (size_t)l * a.mmax * x.s_d + h * 64;
      ll_store(dst + 2 * lane, tag, r0 * inv);
      ll_store(dst + 2 * lane + 1, tag, r1 * inv);
    }
  }
  __syncthreads();
  return true;
}

// Final norm + lm_head rows + argmax candidate of this CTA (engine/infer.js:240-287); GPT-2
// penalties use the generated ids gen_ids[0..n_past).  Publishes the candidate and closes the
// forward with the all-CTA exchange; returns the argmax (same in every CTA) or -1 on a timeout.
template <int NWJ>
__device__ __noinline__ int lm_head(const RunArgs& a, const Lay& S, uint32_t tag, int parity, bool pen,
                                    const int* gen_ids, int n_past, float* logits) {
  const ModelDev& md = a.m;
  const ExchangeDev& x = a.x;
  const int D = md.D, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = gridDim.x, NW = G * kWarps, gw = blockIdx.x * kWarps + warp;
  const int nwords = D >> 3;
  const uint64_t limit = a.wait_ns ? a.wait_ns : kWaitNs;
  constexpr int kG = 4;
  const bool resident = a.lm_rpc > 0;
  Row<NWJ> rw[kG];
  if (!resident) {
#pragma unroll
    for (int g = 0; g < kG; ++g)
      if (gw + g * NW < md.vocab) rw[g].load(md.lm, gw + g * NW, nwords, lane);
  }
  {
    float gv[4], bv[4];
    load_gains(md.norm_f, D, md.arch == 1, gv, bv);
    if (!poll_vec(x.x2 + (size_t)(md.n_layers - 1) * a.mmax * x.s_d, S.xs, D, tag, a.err, limit, a.poll_sleep_ns)) return -1;
    norm_row(S.xs, S.act, S.red, D, md.arch == 1, gv[0], gv[1], gv[2], gv[3], bv[0], bv[1], bv[2], bv[3]);
  }
  int nban = 0, nrec = 0;
  if (pen) {
    if (threadIdx.x == 0) S.misc[0] = 0;
    __syncthreads();
    if (n_past >= 2) {
      const int t1 = gen_ids[n_past - 2], t2 = gen_ids[n_past - 1];
      for (int k = threadIdx.x; k < n_past - 2; k += kThreads)
        if (gen_ids[k] == t1 && gen_ids[k + 1] == t2) S.pen[atomicAdd(&S.misc[0], 1)] = gen_ids[k + 2];
    }
    __syncthreads();
    nban = S.misc[0];
    const int rwin = max(0, n_past - 32);
    nrec = n_past - rwin;
    for (int k = threadIdx.x; k < nrec; k += kThreads) S.pen[nban + k] = gen_ids[rwin + k];
    __syncthreads();
  }
  double best = -INFINITY;
  int bidx = 0x7fffffff;
  // this lane's activations stay in registers for all of its rows (no shared-memory traffic per row)
  float xr[NWJ][8];
#pragma unroll
  for (int j = 0; j < NWJ; ++j) {
    const int k = lane + 32 * j;
#pragma unroll
    for (int e = 0; e < 8; ++e) xr[j][e] = k < nwords ? S.act[8 * k + e] : 0.f;
  }
  auto consider = [&](int r, float v) {
    if (logits && lane == 0) logits[r] = v;
    double val = v;
    if (pen) {
      bool banned = false, recent = false;
      for (int k = lane; k < nban; k += 32) banned |= S.pen[k] == r;
      for (int k = lane; k < nrec; k += 32) recent |= S.pen[nban + k] == r;
      banned = __any_sync(0xffffffffu, banned);
      recent = __any_sync(0xffffffffu, recent);
      if (banned) val = -1e9;
      if (recent && val > -1e8) val = val > 0 ? val / 1.15 : val * 1.15;
    }
    if (val > best) {  // rows rise within a warp: strict > keeps the lowest index on ties
      best = val;
      bidx = r;
    }
  };
  if (resident) {
    // rows [blockIdx.x * lm_rpc, +lm_rpc) from shared memory, warp w takes rows w, w + 8, ...; kRG rows
    // (r, r + 8, ...) per pass, their warp reductions interleaved (same shuffle order as warp_sum), then
    // considered in row order.  Two rows measured best across the three model shapes (four: PetitGPT
    // -1 %, GPT-2 and SmolLM2-360M +0.7 %).
    const int r0 = blockIdx.x * a.lm_rpc, r1 = min(md.vocab, r0 + a.lm_rpc);
    const int ng = nwords >> 2;
    constexpr int kRG = 2;
    for (int r = r0 + warp; r < r1; r += kRG * kWarps) {
      float acc[kRG];
#pragma unroll
      for (int q = 0; q < kRG; ++q) {
        acc[q] = 0.f;
        const int rq = r + q * kWarps;
        if (rq >= r1) continue;
        const uint32_t* wr = S.lmw + (size_t)(rq - r0) * nwords;
        const float* sr = S.lms + (size_t)(rq - r0) * ng;
#pragma unroll
        for (int j = 0; j < NWJ; ++j) {
          const int k = lane + 32 * j;
          if (k < nwords) {
            const uint32_t w = wr[k];
            const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
            float t = nib_at(lo, 0) * xr[j][0];
            t = fmaf(nib_at(hi, 0), xr[j][1], t);
            t = fmaf(nib_at(lo, 1), xr[j][2], t);
            t = fmaf(nib_at(hi, 1), xr[j][3], t);
            t = fmaf(nib_at(lo, 2), xr[j][4], t);
            t = fmaf(nib_at(hi, 2), xr[j][5], t);
            t = fmaf(nib_at(lo, 3), xr[j][6], t);
            t = fmaf(nib_at(hi, 3), xr[j][7], t);
            acc[q] = fmaf(t, sr[k >> 2], acc[q]);
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int q = 0; q < kRG; ++q) acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], o);
#pragma unroll
      for (int q = 0; q < kRG; ++q)
        if (r + q * kWarps < r1) consider(r + q * kWarps, acc[q]);
    }
  } else {
    for (int r0 = gw; r0 < md.vocab; r0 += kG * NW) {
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const int r = r0 + g * NW;
        if (r >= md.vocab) break;
        const float v = rw[g].dot_reg(xr, nwords, lane);
        const int rn = r + kG * NW;  // next group's row for this slot
        if (rn < md.vocab) rw[g].load(md.lm, rn, nwords, lane);
        consider(r, v);
      }
    }
  }
  if (lane == 0) {
    S.cval[warp] = best;
    S.cidx[warp] = bidx;
  }
  __threadfence();  // cache rows written in this forward become visible before the candidate
  __syncthreads();
  if (threadIdx.x == 0) {
    double bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int w = 0; w < kWarps; ++w) {
      if (S.cval[w] > bv || (S.cval[w] == bv && S.cidx[w] < bi)) {
        bv = S.cval[w];
        bi = S.cidx[w];
      }
    }
    const uint64_t bits = (uint64_t)__double_as_longlong(bv);
    uint64_t* slot = x.cand + (((size_t)parity * G + blockIdx.x) * a.mmax) * 4;
    ll_store_u32(slot + 0, tag, (uint32_t)bits);
    ll_store_u32(slot + 1, tag, (uint32_t)(bits >> 32));
    ll_store_u32(slot + 2, tag, (uint32_t)bi);
  }
  // all-CTA exchange of candidates (words 0..2 of each CTA's slot)
  {
    const uint64_t* base = x.cand + (size_t)parity * G * a.mmax * 4;
    uint32_t* dst = reinterpret_cast<uint32_t*>(S.act);
    bool ok = true;
    const uint64_t t0 = globaltimer();
    for (int i = threadIdx.x; i < 3 * G && ok; i += kThreads) {
      const uint64_t* src = base + (size_t)(i / 3) * a.mmax * 4 + (i % 3);
      int rounds = 0;
      for (;;) {
        const uint64_t v = ll_load(src);
        if ((uint32_t)(v >> 32) == tag) {
          dst[i] = (uint32_t)v;
          break;
        }
        if (a.poll_sleep_ns) __nanosleep(a.poll_sleep_ns);
        if (((++rounds & 31) == 0) && (*(volatile int*)a.err || globaltimer() - t0 > limit)) {
          atomicCAS(a.err, 0, 1);
          ok = false;
          break;
        }
      }
    }
    if (!__syncthreads_and(ok)) return -1;
    __threadfence();
  }
  if (warp == 0) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(S.act);
    double bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int g = lane; g < G; g += 32) {
      const double v = __longlong_as_double((long long)(((uint64_t)w[3 * g + 1] << 32) | w[3 * g]));
      const int id = (int)w[3 * g + 2];
      if (v > bv || (v == bv && id < bi)) {
        bv = v;
        bi = id;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) S.misc[2] = bi;
  }
  __syncthreads();
  return S.misc[2];
}

// GELU tanh form (engine/infer.js:166-171), fp32.
__device__ __forceinline__ float gelu(float v) {
  return 0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}


// One layer of the single-token forward at position `pos`.
template <int NWJ_D, int NWJ_F, bool SPLIT>
__device__ __noinline__ bool layer(const RunArgs& a, const Lay& S, int l, int pos, uint32_t tag) {
  const ModelDev& md = a.m;
  const ExchangeDev& x = a.x;
  const LayerDev& L = md.layers[l];
  const int D = md.D, FF = md.FF, QKV = md.QKV;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NW = gridDim.x * kWarps, gw = blockIdx.x * kWarps + warp;
  const int rows0 = blockIdx.x * kWarps;  // first row of this CTA in every row-split stage
  const bool gpt2 = md.arch == 1;
  const uint64_t limit = a.wait_ns ? a.wait_ns : kWaitNs;
  const size_t ofs_d = (size_t)l * a.mmax * x.s_d;
  // ---- QKV rows (wait: previous layer's x2, then norm1)
  if (rows0 < QKV) {
    Row<NWJ_D> rw;
    if (gw < QKV) rw.load(L.qkv, gw, D >> 3, lane);
    float gv[4], bv[4];
    load_gains(L.norm1, D, gpt2, gv, bv);
    float inv = 1.f;
    if (!gpt2 && l > 0) {
      if (!poll_x_rms(x.x2 + ofs_d - (size_t)a.mmax * x.s_d, S.xs, S.act, S.red, D, gv[0], gv[1], gv[2], gv[3], tag,
                      a.err, limit, a.poll_sleep_ns))
        return false;
      inv = rms_inv(S.red, D);
    } else {
      if (l > 0 && !poll_vec(x.x2 + ofs_d - (size_t)a.mmax * x.s_d, S.xs, D, tag, a.err, limit, a.poll_sleep_ns)) return false;
      norm_row(S.xs, S.act, S.red, D, gpt2, gv[0], gv[1], gv[2], gv[3], bv[0], bv[1], bv[2], bv[3]);
    }
    uint64_t* dst = x.qkv + (size_t)l * a.mmax * x.s_qkv;
    for (int r = gw; r < QKV; r += NW) {
      if (r != gw) rw.load(L.qkv, r, D >> 3, lane);
      float v = rw.dot(S.act, D >> 3, lane) * inv;
      if (lane == 0) ll_store(dst + r, tag, L.qkv_b ? v + L.qkv_b[r] : v);
    }
    __syncthreads();
  }
  // ---- attention
  {
    // Attention: NH x ns units (head, position split) on the last CTAs, which have the fewest (for the
    // PetitGPT shape, no) QKV rows.  Once one CTA would need kAttnMinRounds or more rounds of 128
    // positions, one split per round (the merge costs an extra exchange, more than one round saves),
    // capped by the grid, kAttnSplits and the room for the merge's partials in S.act.
    int ns = 1;
    if (SPLIT && md.NH <= (int)gridDim.x) {
      ns = (pos + kAttnRound) / kAttnRound;
      ns = ns >= kAttnMinRounds ? min(ns, kAttnSplits) : 1;
      ns = min(ns, min((int)gridDim.x / md.NH, (act_width(md, gridDim.x) - 256) / kAttnPartWords));
      ns = max(ns, 1);
    }
    const int h0 = md.NH <= (int)gridDim.x ? (int)gridDim.x - md.NH * ns : 0;
    for (int u = (int)blockIdx.x - h0; u >= 0 && u < md.NH * ns; u += gridDim.x)
      if (!attention<SPLIT>(a, S, l, SPLIT ? (u / ns) | ((u % ns) << 8) | (ns << 16) : u, pos, tag)) return false;
  }
  // ---- proj rows + residual (x1)
  if (rows0 < D) {
    Row<NWJ_D> rw;
    if (gw < D) rw.load(L.proj, gw, D >> 3, lane);
    if (!poll_vec(x.att + ofs_d, S.act, D, tag, a.err, limit, a.poll_sleep_ns)) return false;
    for (int r = gw; r < D; r += NW) {
      if (r != gw) rw.load(L.proj, r, D >> 3, lane);
      float v = rw.dot(S.act, D >> 3, lane);
      if (lane == 0) {
        if (L.proj_b) v += L.proj_b[r];
        ll_store(x.x1 + ofs_d + r, tag, S.xs[r] + v);
      }
    }
    __syncthreads();
  }
  // ---- w1/w3 rows + SiLU*mul, or fc + bias + GELU (wait: x1, then norm2).  A warp's first two rows
  // (pairs) are requested before the wait.
  if (rows0 < FF) {
    Row<NWJ_D> r1, r3, r1b, r3b;
    const int gw2 = gw + NW;
    if (gw < FF) {
      r1.load(L.w1, gw, D >> 3, lane);
      if (!gpt2) r3.load(L.w3, gw, D >> 3, lane);
    }
    if (gw2 < FF) {
      r1b.load(L.w1, gw2, D >> 3, lane);
      if (!gpt2) r3b.load(L.w3, gw2, D >> 3, lane);
    }
    float gv[4], bv[4];
    load_gains(L.norm2, D, gpt2, gv, bv);
    float inv = 1.f;
    if (!gpt2) {
      if (!poll_x_rms(x.x1 + ofs_d, S.xs, S.act, S.red, D, gv[0], gv[1], gv[2], gv[3], tag, a.err, limit,
                      a.poll_sleep_ns))
        return false;
      inv = rms_inv(S.red, D);
    } else {
      if (!poll_vec(x.x1 + ofs_d, S.xs, D, tag, a.err, limit, a.poll_sleep_ns)) return false;
      norm_row(S.xs, S.act, S.red, D, gpt2, gv[0], gv[1], gv[2], gv[3], bv[0], bv[1], bv[2], bv[3]);
    }
    uint64_t* dst = x.a + (size_t)l * a.mmax * x.s_ff;
    auto emit = [&](int r, const Row<NWJ_D>& ra, const Row<NWJ_D>& rb) {
      const float u = ra.dot(S.act, D >> 3, lane) * inv;
      if (!gpt2) {
        const float v = rb.dot(S.act, D >> 3, lane) * inv;
        if (lane == 0) ll_store(dst + r, tag, (u / (1.f + expf(-u))) * v);
      } else if (lane == 0) {
        ll_store(dst + r, tag, gelu(L.fc_b ? u + L.fc_b[r] : u));
      }
    };
    if (gw < FF) emit(gw, r1, r3);
    if (gw2 < FF) emit(gw2, r1b, r3b);
    for (int r = gw + 2 * NW; r < FF; r += NW) {
      r1.load(L.w1, r, D >> 3, lane);
      if (!gpt2) r3.load(L.w3, r, D >> 3, lane);
      emit(r, r1, r3);
    }
    __syncthreads();
  } else if (rows0 < D) {
    if (!poll_vec(x.x1 + ofs_d, S.xs, D, tag, a.err, limit, a.poll_sleep_ns)) return false;
  }
  // ---- w2 rows + residual (x2)
  if (rows0 < D) {
    Row<NWJ_F> rw;
    if (gw < D) rw.load(L.w2, gw, FF >> 3, lane);
    if (!poll_vec(x.a + (size_t)l * a.mmax * x.s_ff, S.act, FF, tag, a.err, limit, a.poll_sleep_ns)) return false;
    for (int r = gw; r < D; r += NW) {
      if (r != gw) rw.load(L.w2, r, FF >> 3, lane);
      float v = rw.dot(S.act, FF >> 3, lane);
      if (lane == 0) {
        if (L.mproj_b) v += L.mproj_b[r];
        ll_store(x.x2 + ofs_d + r, tag, S.xs[r] + v);
      }
    }
    __syncthreads();
  }
  return true;
}

}  // namespace d1

// The greedy decode loop on the single-token kernel.  Resumes after a prefill launch: the prompt
// is a.ids[0..n_ids) and out_ids[0..start_gen) already holds the generated ids.  MODE_FORWARD runs
// one forward of a.ids[0] at a.pos0 (forwardDecode).
template <int NWJ_D, int NWJ_F, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) decode1_kernel(const __grid_constant__ RunArgs a) {
  extern __shared__ __align__(16) float smem[];
  const ModelDev& md = a.m;
  d1::Lay S = d1::layout(md, smem);
  if (a.lm_rpc > 0) {
    // this CTA's lm_head rows stay in shared memory for every forward of the launch
    d1::lm_resident_ptrs(md, a.lm_rpc, S);
    const int r0 = blockIdx.x * a.lm_rpc, nr = max(0, min(md.vocab, r0 + a.lm_rpc) - r0);
    const int nwords = md.D >> 3, ng = md.D >> 5;
    const uint4* src = reinterpret_cast<const uint4*>(md.lm.w + (size_t)r0 * nwords);
    uint4* dst = reinterpret_cast<uint4*>(S.lmw);
    for (int i = threadIdx.x; i < nr * nwords / 4; i += kThreads) dst[i] = __ldg(src + i);
    for (int i = threadIdx.x; i < nr * ng; i += kThreads) S.lms[i] = __ldg(md.lm.s + (size_t)r0 * ng + i);
    __syncthreads();
  }
  const bool lead = blockIdx.x == 0 && threadIdx.x == 0;
  const int n = a.n_ids, D = md.D;
  const bool gen_mode = a.mode == MODE_GENERATE;
  if (a.mode == MODE_SELFTEST_WAIT) {
    // Failure-detection self-test: every CTA waits for a candidate word with a tag that no CTA
    // writes in this launch; the wait runs out its limit, raises the error flag and returns.
    d1::poll_vec(a.x.cand + (size_t)blockIdx.x * a.mmax * 4, S.act, 1, a.base_tag, a.err,
                 a.wait_ns ? a.wait_ns : kWaitNs);
    return;
  }
  if (!gen_mode && a.mode != MODE_FORWARD) return;
  int gen = 0, tok = 0, stop = 1, f = 0;
  if (gen_mode) {
    if (*(volatile int*)a.err) return;
    for (int t = threadIdx.x; t < n; t += kThreads) S.hist[t] = a.ids[t];
    for (int t = threadIdx.x; t < a.start_gen; t += kThreads) S.hist[n + t] = a.out_ids[t];
    __syncthreads();
    gen = a.start_gen;
    tok = S.hist[n + gen - 1];
    if (tok == a.eos) stop = 0;
  }
  for (;;) {
    int pos;
    if (gen_mode) {
      // engine/infer.js:625-628
      if (stop == 0 || gen >= a.max_new || n + gen >= md.kv_len) break;
      pos = n + gen - 1;
    } else {
      if (f == 1) break;
      tok = a.ids[0];
      pos = a.pos0;
    }
    const uint32_t tag = a.base_tag + f;
    // embed (engine/infer.js:360-420): dequantised tied lm_head row, GPT-2 /scale_factors + wpe
    {
      const uint8_t* row = reinterpret_cast<const uint8_t*>(md.lm.w) + (size_t)tok * (D / 2);
      const float* sc = md.lm.s + (size_t)tok * (D / 32);
      for (int k = threadIdx.x; k < D; k += kThreads) {
        const int b = row[k >> 1];
        float v = (float)(((k & 1) ? (b >> 4) : (b & 15)) - 8) * sc[k >> 5];
        if (md.arch == 1) {
          if (md.sf) v = __fdiv_rn(v, md.sf[k]);
          v += md.wpe[(size_t)min(pos, md.max_seq - 1) * D + k];
        }
        S.xs[k] = v;
      }
      __syncthreads();
    }
    for (int l = 0; l < md.n_layers; ++l)
      if (!d1::layer<NWJ_D, NWJ_F, SPLIT>(a, S, l, pos, tag)) return;
    const int next = d1::lm_head<NWJ_D>(a, S, tag, f & 1, gen_mode && md.arch == 1, S.hist + n, gen,
                                          gen_mode ? nullptr : a.logits);
    if (next < 0) return;
    ++f;
    if (!gen_mode) {
      if (lead && a.argmax_out) a.argmax_out[0] = next;
      continue;
    }
    tok = next;
    if (lead) {
      a.out_ids[gen] = tok;
      stream_publish(a.stream_ids, gen, tok, 1);
    }
    if (threadIdx.x == 0) S.hist[n + gen] = tok;
    ++gen;
    __syncthreads();
    if (tok == a.eos) stop = 0;
  }
  if (lead) {
    if (gen_mode) {
      a.status[ST_NGEN] = gen;
      a.status[ST_STOP] = stop;
    }
    a.status[ST_FORWARDS] += f;
    const uint64_t t = globaltimer();
    a.status[ST_TEND] = (int32_t)(uint32_t)t;
    a.status[ST_TEND + 1] = (int32_t)(uint32_t)(t >> 32);
  }
}

size_t decode1_smem_bytes(const ModelDev& md, int grid, int lm_rpc) {
  int actw = std::max(std::max(md.D, md.QKV), md.FF);
  actw = std::max(actw, 3 * grid + 4);
  actw = (actw + 3) & ~3;
  size_t words = (size_t)md.D + actw + kWarps * 68 + 2 * kWarps + (md.kv_len + 64) + (md.kv_len + 128) + 32;
  words = (words + 1) & ~(size_t)1;
  words += 2 * kWarps + kWarps;
  words = (words + 3) & ~(size_t)3;
  if (lm_rpc > 0) words += (((size_t)lm_rpc * (md.D >> 3) + 3) & ~(size_t)3) + (size_t)lm_rpc * (md.D >> 5);
  return words * 4;
}

typedef void (*DecodeFn)(const RunArgs);

// split: the variant whose attention splits long contexts over several CTAs per head.
DecodeFn pick_decode1_kernel(int D, int FF, bool split) {
  const int nd = (D / 8 + 31) / 32, nf = (FF / 8 + 31) / 32;
#ifndef MLLM_FAST_BUILD
  if (nd <= 1 && nf <= 2) return split ? decode1_kernel<1, 2, true> : decode1_kernel<1, 2, false>;
#endif
  if (nd <= 3 && nf <= 6) return split ? decode1_kernel<3, 6, true> : decode1_kernel<3, 6, false>;
#ifndef MLLM_FAST_BUILD
  if (nd <= 3 && nf <= 12) return split ? decode1_kernel<3, 12, true> : decode1_kernel<3, 12, false>;
  if (nd <= 4 && nf <= 10) return split ? decode1_kernel<4, 10, true> : decode1_kernel<4, 10, false>;
  if (nd <= 4 && nf <= 16) return split ? decode1_kernel<4, 16, true> : decode1_kernel<4, 16, false>;
#endif
  return nullptr;
}

}  // namespace mllm
