// Persistent decode kernel: prefill, greedy decode, penalised GPT-2 argmax and prompt-lookup
// speculation in ONE cooperative launch (one CTA per SM).
//
// Per forward of M tokens (positions pos0 .. pos0+M-1), per layer, five stages:
//   QKV  : rows of blocks.l.attn.qkv over warps            -> exchange `qkv`
//   ATT  : one CTA per (head, token row): RoPE, KV write, causal attention over the cache
//                                                           -> exchange `att`
//   PROJ : rows of attn.proj + residual                     -> exchange `x1` (all CTAs read it)
//   F1   : rows of w1 and w3 + SiLU*mul (GPT-2: fc + bias + GELU) -> exchange `a`
//   F2   : rows of w2 + residual                            -> exchange `x2`
// then final norm + lm_head rows + argmax, and an all-CTA exchange of per-CTA argmax candidates that
// also closes the forward.  A value crosses CTAs as an 8-byte word {tag, f32}; the consumer spins on
// the tag, with a time limit (device_common.cuh).
//
// Reference semantics (paths relative to the reference project root):
//   engine/infer.js:88-116 gemvQ4, 134-164 rmsNorm/layerNorm, 166-183 GELU/SiLU, 185-225 RoPE,
//   422-504 attention, 506-527 ffn, 240-287 argmax/argmaxGpt2, 553-646 forward/generate;
//   engine/webgpu.js:846-865 lookupDraft and 1239-1270 the verify/accept loop.
// Arithmetic: Q4 dot products accumulate in fp32 (the build's stated tolerance: logits within 2e-2
// of the f64-accumulating CPU path); norms, RoPE, SiLU and GELU are evaluated in f64 as the
// JavaScript does and rounded to f32 where it stores into a Float32Array.
#include <cuda_runtime.h>

#include <algorithm>

#include "device_common.cuh"
#include "engine.cuh"

namespace mllm {

enum LmMode { LM_NONE = 0, LM_LAST = 1, LM_EACH = 2 };

// Weights of one Q4 row for one lane, loaded ahead of the wait for the stage's input.
template <int NWJ>
struct RowW {
  uint32_t w[NWJ];
  float s[NWJ];
  __device__ __forceinline__ void load(const Q4& q, int row, int nwords, int lane, uint64_t pol = 0) {
    const uint32_t* wr = q.w + (size_t)row * nwords;
    const float* sr = q.s + (size_t)row * (nwords >> 2);
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      if (k < nwords) {
        if (pol) {
          w[j] = ld_hint_u32(wr + k, pol);
          s[j] = __uint_as_float(ld_hint_u32(reinterpret_cast<const uint32_t*>(sr) + (k >> 2), pol));
        } else {
          w[j] = ldv_u32(wr + k);
          s[j] = ldv_f32(sr + (k >> 2));
        }
      } else {
        w[j] = 0x88888888u;
        s[j] = 0.f;
      }
    }
  }
  // out[i] = row . x[i] for i < mcount (x rows ld apart), reduced over the warp.
  template <int MT>
  __device__ __forceinline__ void dot(const float* x, int ld, int mcount, int nwords, int lane, float (&out)[MT]) const {
    float acc[MT];
#pragma unroll
    for (int i = 0; i < MT; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      if (k < nwords) {
        if (MT == 1) {
          acc[0] = fmaf(word_dot(w[j], x + 8 * k), s[j], acc[0]);
        } else {
          const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
          float q[8];
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            q[2 * b] = nib_at(lo, b);
            q[2 * b + 1] = nib_at(hi, b);
          }
#pragma unroll
          for (int i = 0; i < MT; ++i) {
            if (i < mcount) {
              const float* xi = x + (size_t)i * ld + 8 * k;
              const float4 xa = *reinterpret_cast<const float4*>(xi);
              const float4 xb = *reinterpret_cast<const float4*>(xi + 4);
              float t = q[0] * xa.x;
              t = fmaf(q[1], xa.y, t);
              t = fmaf(q[2], xa.z, t);
              t = fmaf(q[3], xa.w, t);
              t = fmaf(q[4], xb.x, t);
              t = fmaf(q[5], xb.y, t);
              t = fmaf(q[6], xb.z, t);
              t = fmaf(q[7], xb.w, t);
              acc[i] = fmaf(t, s[j], acc[i]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < MT; ++i) out[i] = warp_sum(acc[i]);
  }
};

// Shared-memory carve-up (all offsets in 4-byte words).
struct Smem {
  float* xs;      // [mmax][D]     residual stream
  float* act;     // [mmax][actw]  stage input / normalised rows / scratch
  float* wpart;   // [kWarps][68]  attention partials
  int* hist;      // [hist_cap]    prompt + generated ids
  int* toks;      // [mmax]        ids of the current forward
  int* res;       // [mmax]        argmax per lm row
  int* pen;       // [hist_cap + 64] GPT-2 banned / recent ids
  int* misc;      // [32]
  double* cval;   // [kWarps][mmax] candidate values
  int* cidx;      // [kWarps][mmax]
  double* red;    // [2][kWarps][16] floats of norm partial sums (double-aligned)
};

struct Ctx {
  const RunArgs& a;
  Smem sm;
  Waiter wt;
  int lane, warp, gw, NW, G, actw, hist_cap;
  uint64_t pol;  // L2 policy for weight loads (0 = default)
  __device__ Ctx(const RunArgs& args) : a(args) {}
};

__device__ __forceinline__ bool cta_has_rows(int rows) { return (int)blockIdx.x * kWarps < rows; }

// L2 prefetch of the rows [r0, r0 + 8) and [r0 + NW, r0 + NW + 8) of a Q4 matrix (the rows this CTA's
// warps own in a GEMV stage) so that the register loads issued before the stage's wait hit L2.
__device__ __forceinline__ void prefetch_rows(const Q4& q, int R, int n, int r0, int NW) {
  for (int base = r0; base < R; base += NW) {
    const int cnt = min(kWarps, R - base);
    prefetch_l2(reinterpret_cast<const uint8_t*>(q.w) + (size_t)base * (n / 2), (uint32_t)cnt * (n / 2));
    prefetch_l2(q.s + (size_t)base * (n / 32), (uint32_t)cnt * (n / 32) * 4);
    if (base + NW >= R) break;
  }
}


// RMSNorm (engine/infer.js:134-143) or LayerNorm (engine/infer.js:147-164) of rows xs[rows_from + i]
// into act[i], i < count.  All 256 threads share every row (element k = thread + 256 j); the gains
// (and LayerNorm biases) are loaded once, in one batch.  fp32 statistics (the JavaScript sums in
// f64; the difference stays at the last-ulp level, well inside the logits tolerance).
struct NormGains {
  float g[4], b[4];
};
__device__ __forceinline__ void load_gains(NormGains& ng, const float* g, int D, bool ln) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int k = threadIdx.x + kThreads * j;
    ng.g[j] = k < D ? ldv_f32(g + k) : 0.f;
    ng.b[j] = (ln && k < D) ? ldv_f32(g + D + k) : 0.f;
  }
}
__device__ __forceinline__ void norm_rows(Ctx& c, const NormGains& ng, int rows_from, int count) {
  const int D = c.a.m.D;
  const bool ln = c.a.m.arch == 1;
  float* red = reinterpret_cast<float*>(c.sm.red);  // [2][kWarps][16]
  for (int i = 0; i < count; ++i) {
    const float* x = c.sm.xs + (size_t)(rows_from + i) * D;
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
    if (c.lane == 0) {
      red[c.warp * 16 + i] = s1;
      red[kWarps * 16 + c.warp * 16 + i] = s2;
    }
  }
  __syncthreads();
  for (int i = 0; i < count; ++i) {
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      s1 += red[w * 16 + i];
      s2 += red[kWarps * 16 + w * 16 + i];
    }
    const float* x = c.sm.xs + (size_t)(rows_from + i) * D;
    float* o = c.sm.act + (size_t)i * c.actw;
    if (!ln) {
      const float inv = 1.f / sqrtf(s2 / D + 1e-6f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = threadIdx.x + kThreads * j;
        if (k < D) o[k] = x[k] * inv * ng.g[j];
      }
    } else {
      const float mean = s1 / D;
      const float var = fmaxf(s2 / D - mean * mean, 0.f);
      const float inv = 1.f / sqrtf(var + 1e-5f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = threadIdx.x + kThreads * j;
        if (k < D) o[k] = fmaf((x[k] - mean) * inv, ng.g[j], ng.b[j]);
      }
    }
  }
  __syncthreads();
}

// Wait for `rows` x `cols` words whose row r starts at rowptr(r); values land in dst[r * dstride + j].
template <class RowPtr>
__device__ __forceinline__ bool poll_gather(Ctx& c, RowPtr rowptr, float* dst, int dstride, int rows, int cols, uint32_t tag) {
  const int n = rows * cols;
  bool ok = true;
  for (int base = threadIdx.x; base < n && ok; base += kThreads * 8) {
    uint32_t pending = 0;
    const uint64_t* src[8];
    int doff[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int i = base + k * kThreads;
      if (i < n) {
        const int r = i / cols, j = i - r * cols;
        src[k] = rowptr(r) + j;
        doff[k] = r * dstride + j;
        pending |= 1u << k;
      } else {
        src[k] = nullptr;
        doff[k] = 0;
      }
    }
    const uint64_t t0 = globaltimer();
    int rounds = 0;
    while (pending) {
      uint64_t v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (pending & (1u << k)) v[k] = ll_load(src[k]);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if ((pending & (1u << k)) && (uint32_t)(v[k] >> 32) == tag) {
          dst[doff[k]] = __uint_as_float((uint32_t)v[k]);
          pending &= ~(1u << k);
        }
      }
      if (pending) {
        if (((++rounds & 31) == 0) && c.wt.give_up(t0)) {
          ok = false;
          break;
        }
        if (c.a.poll_sleep_ns) __nanosleep(c.a.poll_sleep_ns);
      }
    }
  }
  return __syncthreads_and(ok);
}

// GEMV over the rows this warp owns: out(r, i, value) for token rows i < M.  Two rows' weights are
// in flight ahead of use: the first two are requested before `wait()` (which polls the stage input
// and may normalise it), later ones one row ahead of the FMAs.  Ends with a CTA barrier: the next
// stage may overwrite `x`.
template <int NWJ, bool MULTI, class Wait, class Out>
__device__ __forceinline__ bool gemv_stage(Ctx& c, const Q4& q, int R, int n, const float* x, int ld, int M, Wait wait, Out out) {
  const int nwords = n >> 3;
  RowW<NWJ> cur, nxt;
  int r = c.gw;
  if (r < R) cur.load(q, r, nwords, c.lane, c.pol);
  if (r + c.NW < R) nxt.load(q, r + c.NW, nwords, c.lane, c.pol);
  if (!wait()) return false;
  for (; r < R; r += c.NW) {
    if (!MULTI || M == 1) {
      float v[1];
      cur.template dot<1>(x, ld, 1, nwords, c.lane, v);
      out(r, 0, v[0]);
    } else if constexpr (MULTI) {
      for (int m0 = 0; m0 < M; m0 += 4) {
        float v[4];
        cur.template dot<4>(x + (size_t)m0 * ld, ld, M - m0, nwords, c.lane, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) out(r, m0 + i, v[i]);
      }
    }
    cur = nxt;
    if (r + 2 * c.NW < R) nxt.load(q, r + 2 * c.NW, nwords, c.lane, c.pol);
  }
  __syncthreads();
  return true;
}

// Two matrices sharing rows and input (w1 and w3): out(r, i, u, v); same pipelining.
template <int NWJ, bool MULTI, class Wait, class Out>
__device__ __forceinline__ bool gemv2_stage(Ctx& c, const Q4& q1, const Q4& q3, int R, int n, const float* x, int ld, int M, Wait wait,
                            Out out) {
  const int nwords = n >> 3;
  RowW<NWJ> c1, c3, n1, n3;
  int r = c.gw;
  if (r < R) {
    c1.load(q1, r, nwords, c.lane, c.pol);
    c3.load(q3, r, nwords, c.lane, c.pol);
  }
  if (r + c.NW < R) {
    n1.load(q1, r + c.NW, nwords, c.lane, c.pol);
    n3.load(q3, r + c.NW, nwords, c.lane, c.pol);
  }
  if (!wait()) return false;
  for (; r < R; r += c.NW) {
    if (!MULTI || M == 1) {
      float u[1], v[1];
      c1.template dot<1>(x, ld, 1, nwords, c.lane, u);
      c3.template dot<1>(x, ld, 1, nwords, c.lane, v);
      out(r, 0, u[0], v[0]);
    } else if constexpr (MULTI) {
      for (int m0 = 0; m0 < M; m0 += 4) {
        float u[4], v[4];
        c1.template dot<4>(x + (size_t)m0 * ld, ld, M - m0, nwords, c.lane, u);
        c3.template dot<4>(x + (size_t)m0 * ld, ld, M - m0, nwords, c.lane, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) out(r, m0 + i, u[i], v[i]);
      }
    }
    c1 = n1;
    c3 = n3;
    if (r + 2 * c.NW < R) {
      n1.load(q1, r + 2 * c.NW, nwords, c.lane, c.pol);
      n3.load(q3, r + 2 * c.NW, nwords, c.lane, c.pol);
    }
  }
  __syncthreads();
  return true;
}

// Causal attention of one (head, token row) unit (engine/infer.js:422-495 for one q row).
// Layout: 4 lanes per position, 16 dims each, so one K or V row (256 B) is read by one lane quad in a
// single coalesced request; a warp covers 8 positions per step, the CTA 64.  Softmax is online
// (running max / sum per warp), combined across warps at the end.
template <bool MULTI>
__device__ __forceinline__ bool attention_unit(Ctx& c, int l, int h, int m_, int pos0, uint32_t tag) {
  const int m = MULTI ? m_ : 0;
  const ModelDev& md = c.a.m;
  const int D = md.D, NKV = md.NKV, rep = md.NH / md.NKV, kvh = h / rep;
  const int pos_m = pos0 + m, npos = pos_m + 1, nloc = m + 1;
  const ExchangeDev& x = c.a.x;
  float* q = c.sm.act;                 // [64]
  float* kl = c.sm.act + 64;           // [nloc][64]
  float* vl = kl + (size_t)nloc * 64;  // [nloc][64]
  const uint64_t* qkv_l = x.qkv + (size_t)l * c.a.mmax * x.s_qkv;
  // rows: 0 -> q of (h, m); 1..nloc -> k of local rows; nloc+1..2nloc -> v of local rows
  auto rowptr = [&](int r) -> const uint64_t* {
    if (r == 0) return qkv_l + (size_t)m * x.s_qkv + h * kHeadDim;
    if (r <= nloc) return qkv_l + (size_t)(r - 1) * x.s_qkv + D + kvh * kHeadDim;
    return qkv_l + (size_t)(r - 1 - nloc) * x.s_qkv + D + NKV * kHeadDim + kvh * kHeadDim;
  };
  // RoPE table values for this thread's pairs are fetched before the wait (engine/infer.js:208-225).
  const bool rope = md.arch == 0 && md.rope_dim > 0;
  const int half = rope ? md.rope_dim / 2 : 1;
  const int npairs = rope ? (1 + nloc) * half : 0;
  float rc0[3], rc1[3], rs0[3], rs1[3];  // (1 + 16) * 32 pairs / 256 threads <= 3 per thread
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int t = threadIdx.x + kThreads * j;
    if (t < npairs) {
      const int row = t / half, d = t - row * half;
      const int pos = row == 0 ? pos_m : pos0 + row - 1;
      const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
      const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
      rc0[j] = ldv_f32(cs + d);
      rc1[j] = ldv_f32(cs + d + half);
      rs0[j] = ldv_f32(sn + d);
      rs1[j] = ldv_f32(sn + d + half);
    }
  }
  if (!poll_gather(c, rowptr, q, 64, 1 + 2 * nloc, 64, tag)) return false;
  if (rope) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int t = threadIdx.x + kThreads * j;
      if (t < npairs) {
        const int row = t / half, d = t - row * half;
        float* v = row == 0 ? q : kl + (size_t)(row - 1) * 64;
        const float a0 = v[d], a1 = v[d + half];
        v[d] = fmaf(-a1, rs0[j], a0 * rc0[j]);
        v[d + half] = fmaf(a0, rs1[j], a1 * rc1[j]);
      }
    }
    __syncthreads();
  }
  const size_t kv_base = ((size_t)l * NKV + kvh) * md.kv_len;
  // The first head of each group owns the cache rows of its kv head (engine/infer.js:457-464).
  if (h % rep == 0 && threadIdx.x < 128) {
    const int d = threadIdx.x & 63;
    if (threadIdx.x < 64) c.a.kc[(kv_base + pos_m) * 64 + d] = kl[(size_t)m * 64 + d];
    else c.a.vc[(kv_base + pos_m) * 64 + d] = vl[(size_t)m * 64 + d];
  }
  const int qd = c.lane & 3, pg = c.lane >> 2;
  float qv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) qv[i] = q[qd * 16 + i];
  float mrun = -INFINITY, lrun = 0.f, o[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i] = 0.f;
  for (int base = c.warp * 8; base < npos; base += kWarps * 8) {
    const int p = base + pg;
    const bool valid = p < npos;
    float4 kk[4], vv[4];
    if (valid && p < pos0) {
      const float* kr = c.a.kc + (kv_base + p) * 64 + qd * 16;
      const float* vr = c.a.vc + (kv_base + p) * 64 + qd * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) kk[j] = ldcg_f4(kr + 4 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j) vv[j] = ldcg_f4(vr + 4 * j);
    } else if (valid) {
      const float* kr = kl + (size_t)(p - pos0) * 64 + qd * 16;
      const float* vr = vl + (size_t)(p - pos0) * 64 + qd * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kk[j] = *reinterpret_cast<const float4*>(kr + 4 * j);
        vv[j] = *reinterpret_cast<const float4*>(vr + 4 * j);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) kk[j] = vv[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float part = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      part = fmaf(qv[4 * j], kk[j].x, part);
      part = fmaf(qv[4 * j + 1], kk[j].y, part);
      part = fmaf(qv[4 * j + 2], kk[j].z, part);
      part = fmaf(qv[4 * j + 3], kk[j].w, part);
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    const float sc = valid ? part * 0.125f : -INFINITY;  // 1/sqrt(64), exact (engine/infer.js:466)
    const float newm = fmaxf(mrun, warp_max(sc));
    const float e = valid ? expf(sc - newm) : 0.f;
    const float corr = mrun == -INFINITY ? 0.f : expf(mrun - newm);
    lrun = fmaf(lrun, corr, warp_sum(qd == 0 ? e : 0.f));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[4 * j] = fmaf(e, vv[j].x, o[4 * j] * corr);
      o[4 * j + 1] = fmaf(e, vv[j].y, o[4 * j + 1] * corr);
      o[4 * j + 2] = fmaf(e, vv[j].z, o[4 * j + 2] * corr);
      o[4 * j + 3] = fmaf(e, vv[j].w, o[4 * j + 3] * corr);
    }
    mrun = newm;
  }
  // sum the 8 position groups (lanes with equal qd)
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    o[i] += __shfl_xor_sync(0xffffffffu, o[i], 4);
    o[i] += __shfl_xor_sync(0xffffffffu, o[i], 8);
    o[i] += __shfl_xor_sync(0xffffffffu, o[i], 16);
  }
  float* wp = c.sm.wpart + c.warp * 68;
  if (c.lane == 0) {
    wp[0] = mrun;
    wp[1] = lrun;
  }
  if (pg == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) wp[4 + qd * 16 + i] = o[i];
  }
  __syncthreads();
  if (c.warp == 0) {
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, c.sm.wpart[w * 68]);
    float L = 0.f, r0 = 0.f, r1 = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float* pw = c.sm.wpart + w * 68;
      if (pw[1] > 0.f) {
        const float f = expf(pw[0] - M);
        L = fmaf(pw[1], f, L);
        r0 = fmaf(pw[4 + 2 * c.lane], f, r0);
        r1 = fmaf(pw[4 + 2 * c.lane + 1], f, r1);
      }
    }
    const float inv = 1.f / L;
    uint64_t* dst = x.att + ((size_t)l * c.a.mmax + m) * x.s_d + h * kHeadDim;
    ll_store(dst + 2 * c.lane, tag, r0 * inv);
    ll_store(dst + 2 * c.lane + 1, tag, r1 * inv);
  }
  __syncthreads();
  return true;
}

// GELU tanh form (engine/infer.js:166-171), fp32.
__device__ __forceinline__ float gelu_new(float v) {
  return 0.5f * v * (1.f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

// One forward over c.sm.toks[0..M) at positions pos0..; returns false when a wait gave up.
// lm: LM_NONE / LM_LAST / LM_EACH.  gpt2_hist (GPT-2 generate): apply argmaxGpt2 penalties using
// the generated ids sm.hist[hist_from .. hist_from + n_past).
template <int NWJ_D, int NWJ_F, bool MULTI>
__device__ __forceinline__ bool forward(Ctx& c, int M_, int pos0, int lm, uint32_t tag, int parity, bool gpt2_pen, int hist_from,
                        int n_past, float* logits_out) {
  const RunArgs& a = c.a;
  const ModelDev& md = a.m;
  const ExchangeDev& x = a.x;
  const int D = md.D, FF = md.FF, QKV = md.QKV, mmax = a.mmax, actw = c.actw;
  const int M = MULTI ? M_ : 1;
  Smem& sm = c.sm;

  // ---- embed (engine/infer.js:360-420): dequantised tied lm_head row, GPT-2 /scale_factors + wpe
  for (int t = threadIdx.x; t < M * D; t += kThreads) {
    const int i = t / D, k = t % D;
    const int id = sm.toks[i];
    const uint8_t* row = reinterpret_cast<const uint8_t*>(md.lm.w) + (size_t)id * (D / 2);
    const int b = row[k >> 1];
    const int qv = (k & 1) ? (b >> 4) : (b & 15);
    float v = (float)(qv - 8) * md.lm.s[(size_t)id * (D / 32) + (k >> 5)];
    if (md.arch == 1) {
      if (md.sf) v = __fdiv_rn(v, md.sf[k]);
      const int pos = min(pos0 + i, md.max_seq - 1);
      v = v + md.wpe[(size_t)pos * D + k];
    }
    sm.xs[(size_t)i * D + k] = v;
  }
  __syncthreads();

  auto poll_rowsof = [&](const uint64_t* src, int stride, float* dst, int dstride, int cols) {
    return poll_gather(c, [&](int r) { return src + (size_t)r * stride; }, dst, dstride, M, cols, tag);
  };
  for (int l = 0; l < md.n_layers; ++l) {
    const LayerDev& L = md.layers[l];
    if (threadIdx.x == 0 && c.a.l2_prefetch) {
      if (l + 1 < md.n_layers) {
        const LayerDev& Ln = md.layers[l + 1];
        const int r0 = blockIdx.x * kWarps;
        prefetch_rows(Ln.qkv, QKV, D, r0, c.NW);
        prefetch_rows(Ln.proj, D, D, r0, c.NW);
        prefetch_rows(Ln.w1, FF, D, r0, c.NW);
        if (md.arch == 0) prefetch_rows(Ln.w3, FF, D, r0, c.NW);
        prefetch_rows(Ln.w2, D, FF, r0, c.NW);
      }
      // K/V rows this CTA's attention unit will read (positions < pos0 of its kv head)
      if ((int)blockIdx.x < md.NH && pos0 > 0) {
        const int kvh = blockIdx.x / (md.NH / md.NKV);
        const size_t kv_base = ((size_t)l * md.NKV + kvh) * md.kv_len;
        prefetch_l2(c.a.kc + kv_base * 64, (uint32_t)pos0 * 256);
        prefetch_l2(c.a.vc + kv_base * 64, (uint32_t)pos0 * 256);
      }
    }
    const uint64_t* x2_prev = l > 0 ? x.x2 + (size_t)(l - 1) * mmax * x.s_d : nullptr;
    // ---------------- QKV (waits for the previous layer's x2 when the CTA needs the residual stream)
    if (cta_has_rows(QKV)) {
      uint64_t* dst = x.qkv + (size_t)l * mmax * x.s_qkv;
      const float* bias = L.qkv_b;
      NormGains ng;
      load_gains(ng, L.norm1, D, md.arch == 1);
      auto wait = [&] {
        if (x2_prev && !poll_rowsof(x2_prev, x.s_d, sm.xs, D, D)) return false;
        norm_rows(c, ng, 0, M);
        return true;
      };
      if (!gemv_stage<NWJ_D, MULTI>(c, L.qkv, QKV, D, sm.act, actw, M, wait, [&](int r, int i, float v) {
            if (c.lane == 0) ll_store(dst + (size_t)i * x.s_qkv + r, tag, bias ? v + bias[r] : v);
          }))
        return false;
    } else if (x2_prev && cta_has_rows(D)) {
      if (!poll_rowsof(x2_prev, x.s_d, sm.xs, D, D)) return false;
    }
    // ---------------- ATT
    for (int u = blockIdx.x; u < md.NH * M; u += c.G) {
      if (!attention_unit<MULTI>(c, l, u % md.NH, u / md.NH, pos0, tag)) return false;
    }
    // ---------------- PROJ + residual
    if (cta_has_rows(D)) {
      const uint64_t* src = x.att + (size_t)l * mmax * x.s_d;
      uint64_t* dst = x.x1 + (size_t)l * mmax * x.s_d;
      const float* bias = L.proj_b;
      auto wait = [&] { return poll_rowsof(src, x.s_d, sm.act, actw, D); };
      if (!gemv_stage<NWJ_D, MULTI>(c, L.proj, D, D, sm.act, actw, M, wait, [&](int r, int i, float v) {
            if (c.lane == 0) {
              const float y = bias ? v + bias[r] : v;
              ll_store(dst + (size_t)i * x.s_d + r, tag, sm.xs[(size_t)i * D + r] + y);
            }
          }))
        return false;
    }
    // ---------------- F1: w1/w3 + SiLU*mul, or fc + bias + GELU (waits for x1)
    const uint64_t* x1_l = x.x1 + (size_t)l * mmax * x.s_d;
    if (cta_has_rows(FF)) {
      uint64_t* dst = x.a + (size_t)l * mmax * x.s_ff;
      NormGains ng;
      load_gains(ng, L.norm2, D, md.arch == 1);
      auto wait = [&] {
        if (!poll_rowsof(x1_l, x.s_d, sm.xs, D, D)) return false;
        norm_rows(c, ng, 0, M);
        return true;
      };
      bool ok;
      if (md.arch == 0) {
        ok = gemv2_stage<NWJ_D, MULTI>(c, L.w1, L.w3, FF, D, sm.act, actw, M, wait, [&](int r, int i, float u, float v) {
          if (c.lane == 0) ll_store(dst + (size_t)i * x.s_ff + r, tag, (u / (1.f + expf(-u))) * v);
        });
      } else {
        const float* bias = L.fc_b;
        ok = gemv_stage<NWJ_D, MULTI>(c, L.w1, FF, D, sm.act, actw, M, wait, [&](int r, int i, float v) {
          if (c.lane == 0) ll_store(dst + (size_t)i * x.s_ff + r, tag, gelu_new(bias ? v + bias[r] : v));
        });
      }
      if (!ok) return false;
    } else if (cta_has_rows(D)) {
      if (!poll_rowsof(x1_l, x.s_d, sm.xs, D, D)) return false;
    }
    // ---------------- F2: w2 + residual
    if (cta_has_rows(D)) {
      const uint64_t* src = x.a + (size_t)l * mmax * x.s_ff;
      uint64_t* dst = x.x2 + (size_t)l * mmax * x.s_d;
      const float* bias = L.mproj_b;
      auto wait = [&] { return poll_rowsof(src, x.s_ff, sm.act, actw, FF); };
      if (!gemv_stage<NWJ_F, MULTI>(c, L.w2, D, FF, sm.act, actw, M, wait, [&](int r, int i, float v) {
            if (c.lane == 0) {
              const float y = bias ? v + bias[r] : v;
              ll_store(dst + (size_t)i * x.s_d + r, tag, sm.xs[(size_t)i * D + r] + y);
            }
          }))
        return false;
    }
  }
  const uint64_t* x2_last = x.x2 + (size_t)(md.n_layers - 1) * mmax * x.s_d;

  // ---------------- final norm + lm_head + argmax candidates
  const int nlm = (MULTI && lm == LM_EACH) ? M : 1;
  const int lm_from = lm == LM_EACH ? 0 : M - 1;
  if (lm != LM_NONE) {
    NormGains ng;
    load_gains(ng, md.norm_f, D, md.arch == 1);
    if (!poll_rowsof(x2_last, x.s_d, sm.xs, D, D)) return false;
    norm_rows(c, ng, lm_from, nlm);
    // GPT-2 penalties (engine/infer.js:252-287): banned next ids after the last bigram, and the
    // recent-window ids that get the 1.15 repetition penalty.
    int nban = 0, nrec = 0;
    if (gpt2_pen) {
      if (threadIdx.x == 0) sm.misc[0] = 0;
      __syncthreads();
      const int* h = sm.hist + hist_from;
      if (n_past >= 2) {
        const int t1 = h[n_past - 2], t2 = h[n_past - 1];
        for (int k = threadIdx.x; k < n_past - 2; k += kThreads)
          if (h[k] == t1 && h[k + 1] == t2) sm.pen[atomicAdd(&sm.misc[0], 1)] = h[k + 2];
      }
      __syncthreads();
      nban = sm.misc[0];
      const int rw = max(0, n_past - 32);
      nrec = n_past - rw;
      for (int k = threadIdx.x; k < nrec; k += kThreads) sm.pen[nban + k] = h[rw + k];
      __syncthreads();
    }
    double best[4];
    int bidx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      best[i] = -INFINITY;
      bidx[i] = 0x7fffffff;
    }
    const int nwords = D >> 3;
    constexpr int kGroup = 8;  // rows whose weights are in flight together
    RowW<NWJ_D> rw[kGroup];
    // LM rows are processed in tiles of 4 token rows; nlm <= mmax <= 16 -> up to 4 passes.
    for (int m0 = 0; m0 < nlm; m0 += 4) {
      for (int r0 = c.gw; r0 < md.vocab; r0 += kGroup * c.NW) {
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
          const int r = r0 + g * c.NW;
          if (r < md.vocab) rw[g].load(md.lm, r, nwords, c.lane, c.pol);
        }
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
        const int r = r0 + g * c.NW;
        if (r >= md.vocab) break;
        float v[4];
        if (!MULTI || nlm == 1) {
          float v1[1];
          rw[g].template dot<1>(sm.act, actw, 1, nwords, c.lane, v1);
          v[0] = v1[0];
        } else if constexpr (MULTI) {
          rw[g].template dot<4>(sm.act + (size_t)m0 * actw, actw, nlm - m0, nwords, c.lane, v);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (m0 + i >= nlm) break;
          if (logits_out && c.lane == i) logits_out[(size_t)(m0 + i) * md.vocab + r] = v[i];
          double val = v[i];
          if (gpt2_pen) {
            bool banned = false, recent = false;
            for (int k = c.lane; k < nban; k += 32) banned |= sm.pen[k] == r;
            for (int k = c.lane; k < nrec; k += 32) recent |= sm.pen[nban + k] == r;
            banned = __any_sync(0xffffffffu, banned);
            recent = __any_sync(0xffffffffu, recent);
            if (banned) val = -1e9;
            if (recent && val > -1e8) val = val > 0 ? val / 1.15 : val * 1.15;
          }
          if (val > best[i]) {
            best[i] = val;
            bidx[i] = r;
          }
        }
        }
      }
      // CTA-level reduction of this tile
      if (c.lane == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          c.sm.cval[c.warp * 4 + i] = best[i];
          c.sm.cidx[c.warp * 4 + i] = bidx[i];
        }
      }
      __threadfence();  // cache rows written in this forward become visible before the candidate
      __syncthreads();
      if (threadIdx.x < 4 && m0 + (int)threadIdx.x < nlm) {
        const int i = threadIdx.x;
        double bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kWarps; ++w) {
          const double v = c.sm.cval[w * 4 + i];
          const int id = c.sm.cidx[w * 4 + i];
          if (v > bv || (v == bv && id < bi)) {
            bv = v;
            bi = id;
          }
        }
        const uint64_t bits = (uint64_t)__double_as_longlong(bv);
        uint64_t* slot = x.cand + (((size_t)parity * c.G + blockIdx.x) * mmax + (m0 + i)) * 4;
        ll_store_u32(slot + 0, tag, (uint32_t)bits);
        ll_store_u32(slot + 1, tag, (uint32_t)(bits >> 32));
        ll_store_u32(slot + 2, tag, (uint32_t)bi);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        best[i] = -INFINITY;
        bidx[i] = 0x7fffffff;
      }
      __syncthreads();
    }
  } else {
    __threadfence();
    if (threadIdx.x == 0) {
      uint64_t* slot = x.cand + (((size_t)parity * c.G + blockIdx.x) * mmax) * 4;
      ll_store_u32(slot + 0, tag, 0);
      ll_store_u32(slot + 1, tag, 0xFFF00000u);  // -inf
      ll_store_u32(slot + 2, tag, 0);
    }
  }
  // ---------------- all-CTA exchange of candidates: closes the forward
  {
    const uint64_t* base = x.cand + (size_t)parity * c.G * mmax * 4;
    float* dst = sm.act;  // [G * nlm][3] raw 32-bit payloads
    if (!poll_gather(c, [&](int r) { return base + ((size_t)(r / nlm) * mmax + (r % nlm)) * 4; }, dst, 3, c.G * nlm, 3,
                     tag))
      return false;
    __threadfence();
    for (int i = c.warp; i < nlm; i += kWarps) {
      double bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int g = c.lane; g < c.G; g += 32) {
        const uint32_t* w = reinterpret_cast<const uint32_t*>(dst) + ((size_t)g * nlm + i) * 3;
        const double v = __longlong_as_double((long long)(((uint64_t)w[1] << 32) | w[0]));
        const int id = (int)w[2];
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
      if (c.lane == 0) sm.res[i] = bi;
    }
    __syncthreads();
  }
  return true;
}

// Largest i < len - n with seq[i .. i+n) == seq[len-n .. len) (engine/webgpu.js:846-865); returns the
// draft length and writes the draft into `out`.  All threads call it; all get the same answer.
__device__ __forceinline__ int lookup_draft(Ctx& c, const int* seq, int len, int k, int n, int* out) {
  if (threadIdx.x == 0) c.sm.misc[1] = -1;
  __syncthreads();
  if (len >= n + 1) {
    const int limit = len - n;
    int best = -1;
    for (int i = threadIdx.x; i < limit; i += kThreads) {
      bool ok = true;
      for (int j = 0; j < n; ++j)
        if (seq[i + j] != seq[len - n + j]) {
          ok = false;
          break;
        }
      if (ok) best = i;
    }
    if (best >= 0) atomicMax(&c.sm.misc[1], best);
  }
  __syncthreads();
  const int i = c.sm.misc[1];
  int d = 0;
  if (i >= 0)
    for (int t = 0; t < k && i + n + t < len; ++t) out[d++] = seq[i + n + t];
  __syncthreads();
  return d;
}

template <int NWJ_D, int NWJ_F, bool MULTI>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ RunArgs a) {
  extern __shared__ __align__(16) float smem[];
  Ctx c(a);
  c.lane = threadIdx.x & 31;
  c.warp = threadIdx.x >> 5;
  c.G = gridDim.x;
  c.gw = blockIdx.x * kWarps + c.warp;
  c.NW = c.G * kWarps;
  c.wt.err = a.err;
  c.wt.limit_ns = a.wait_ns ? a.wait_ns : kWaitNs;
  c.pol = a.weight_policy == 1 ? l2_policy_evict_last() : 0;
  const ModelDev& md = a.m;
  const int mmax = a.mmax;
  const int srows = a.srows;  // token rows held in shared memory (1 for the single-token kernel)
  int actw = max(max(md.D, md.QKV), md.FF);
  actw = max(actw, 3 * c.G * 1 + 4);
  actw = (actw + 3) & ~3;
  c.actw = actw;
  c.hist_cap = md.kv_len + 64;
  {
    float* p = smem;
    c.sm.xs = p; p += (size_t)srows * md.D;
    c.sm.act = p; p += (size_t)srows * actw;
    c.sm.wpart = p; p += kWarps * 68;
    c.sm.hist = reinterpret_cast<int*>(p); p += c.hist_cap;
    c.sm.toks = reinterpret_cast<int*>(p); p += 16;
    c.sm.res = reinterpret_cast<int*>(p); p += 16;
    c.sm.pen = reinterpret_cast<int*>(p); p += c.hist_cap + 64;
    c.sm.misc = reinterpret_cast<int*>(p); p += 32;
    p = reinterpret_cast<float*>(((uintptr_t)p + 7) & ~(uintptr_t)7);
    c.sm.cval = reinterpret_cast<double*>(p); p += 2 * kWarps * 4;
    c.sm.cidx = reinterpret_cast<int*>(p); p += kWarps * 4;
    c.sm.red = reinterpret_cast<double*>(p); p += 2 * kWarps * 16;
  }
  const bool lead = blockIdx.x == 0 && threadIdx.x == 0;
  if (lead && a.start_gen == 0) {
    const uint64_t t = globaltimer();
    a.status[ST_T0] = (int32_t)(uint32_t)t;
    a.status[ST_T0 + 1] = (int32_t)(uint32_t)(t >> 32);
  }
  if (a.mode == MODE_SELFTEST_WAIT) {
    // Failure-detection self-test: every CTA waits for a candidate word with a tag no CTA writes in
    // this launch.  The wait runs out its limit, raises the error flag and the kernel returns; the
    // host reports MLLM_ERR_TIMEOUT and the context stays usable.
    const uint64_t* w = a.x.cand + (size_t)blockIdx.x * mmax * 4;
    poll_gather(c, [&](int) { return w; }, c.sm.act, 1, 1, 1, a.base_tag);
    return;
  }
  // One call site of forward() (so that it inlines and the context stays in registers); a small
  // state machine picks each forward's rows: prompt chunks, then greedy steps or speculative verifies.
  const int n = a.n_ids;
  const bool gen_mode = a.mode == MODE_GENERATE;
  const bool gpt2 = md.arch == 1;
  int* hist = c.sm.hist;
  if (gen_mode) {
    bool bad = false;
    for (int t = threadIdx.x; t < n; t += kThreads) {
      const int id = a.ids[t];
      bad |= id < 0 || id >= md.vocab;
      hist[t] = id;
    }
    if (__syncthreads_or(bad)) {  // device-resident prompts are checked here (error code 2)
      if (threadIdx.x == 0) atomicCAS(a.err, 0, 2);
      return;
    }
  }
  int f = 0;          // forwards run in this launch
  int c0 = 0;         // next prompt chunk
  bool prefill = true;
  int hlen = n, gen = 0, stop = 1 /* max_new_tokens */, hits = 0, tries = 0, tok = 0, cache = 0, dl = 0;
  if (gen_mode && a.start_gen > 0) {
    // Resume after a separate prefill launch: the generated ids so far are in out_ids.
    if (*(volatile int*)a.err) return;
    for (int t = threadIdx.x; t < a.start_gen; t += kThreads) hist[n + t] = a.out_ids[t];
    __syncthreads();
    gen = a.start_gen;
    hlen = n + gen;
    tok = hist[hlen - 1];
    prefill = false;
    cache = n + gen - 1;
    if (tok == a.eos) stop = 0;
  }
  const bool stop_now = gen_mode && a.start_gen > 0 && tok == a.eos;
  int* draft = c.sm.pen;  // speculation is llama-only, so the GPT-2 penalty list is free
  for (; !stop_now;) {
    int M, pos0, lm = LM_LAST, n_past = 0;
    bool pen = false;
    float* lg = nullptr;
    if (!gen_mode || prefill) {
      if (c0 >= n) break;
      M = min(mmax, n - c0);
      const bool last = c0 + M >= n;
      for (int t = threadIdx.x; t < M; t += kThreads) c.sm.toks[t] = gen_mode ? hist[c0 + t] : a.ids[c0 + t];
      if (gen_mode) {
        pos0 = c0;
        lm = last ? LM_LAST : LM_NONE;
        pen = gpt2;  // first id: empty history, no penalty (engine/infer.js:614)
      } else {
        pos0 = a.pos0 + c0;
        lm = a.logits_each ? LM_EACH : (last ? LM_LAST : LM_NONE);
        if (a.logits) lg = a.logits + (size_t)(a.logits_each ? c0 : 0) * md.vocab;
      }
    } else if (MULTI && a.spec_k > 0) {
      // engine/webgpu.js:1239-1249: draft from prompt + accepted ids, verify [last, ...draft]
      if (gen >= a.max_new || cache >= md.kv_len - 1) break;
      pos0 = cache;
      dl = lookup_draft(c, hist, hlen, min(a.spec_k, mmax - 1), a.ngram, draft);
      if (pos0 + dl > md.kv_len - 1) dl = md.kv_len - 1 - pos0;
      ++tries;
      if (threadIdx.x == 0) {
        c.sm.toks[0] = tok;
        for (int i = 0; i < dl; ++i) c.sm.toks[1 + i] = draft[i];
      }
      M = 1 + dl;
      lm = dl > 0 ? LM_EACH : LM_LAST;
    } else {
      // engine/infer.js:625-628
      if (gen >= a.max_new || n + gen >= md.kv_len) break;
      if (threadIdx.x == 0) c.sm.toks[0] = tok;
      M = 1;
      pos0 = n + gen - 1;
      pen = gpt2;
      n_past = gen;
    }
    __syncthreads();
    if (!forward<NWJ_D, NWJ_F, MULTI>(c, M, pos0, lm, a.base_tag + f, f & 1, pen, n, n_past, lg)) return;
    ++f;
    if (!gen_mode) {
      if (lead && a.argmax_out) {
        if (a.logits_each)
          for (int i = 0; i < M; ++i) a.argmax_out[c0 + i] = c.sm.res[i];
        else if (c0 + M >= n)
          a.argmax_out[0] = c.sm.res[0];
      }
      c0 += M;
      continue;
    }
    if (prefill) {
      c0 += M;
      if (c0 < n) continue;
      // first id from the prefill (engine/infer.js:611-616, engine/webgpu.js:1178-1196)
      prefill = false;
      tok = c.sm.res[0];
      cache = n < md.kv_len - 1 ? n : md.kv_len - 1;
      if (lead) {
        a.out_ids[0] = tok;
        const uint64_t t = globaltimer();
        a.status[ST_TFIRST] = (int32_t)(uint32_t)t;
        a.status[ST_TFIRST + 1] = (int32_t)(uint32_t)(t >> 32);
      }
      hist[hlen++] = tok;
      gen = 1;
      if (a.prefill_only) {
        __syncthreads();
        if (tok == a.eos) stop = 0;
        break;
      }
    } else if (MULTI && a.spec_k > 0) {
      // engine/webgpu.js:1249-1268: accept r[0], then r[k+1] while r[k] == draft[k]
      const int r0 = c.sm.res[0];
      if (lead) a.out_ids[gen] = r0;
      hist[hlen++] = r0;
      ++gen;
      cache = pos0 + 1;
      tok = r0;
      if (r0 != a.eos && dl > 0) {
        for (int k = 0; k < dl; ++k) {
          if (c.sm.res[k] != draft[k]) break;
          if (gen >= a.max_new) break;
          const int nxt = c.sm.res[k + 1];
          ++hits;
          if (lead) a.out_ids[gen] = nxt;
          hist[hlen++] = nxt;
          ++gen;
          cache = pos0 + 2 + k;
          tok = nxt;
          if (nxt == a.eos) break;
        }
      }
    } else {
      tok = c.sm.res[0];
      if (lead) a.out_ids[gen] = tok;
      hist[hlen++] = tok;
      ++gen;
    }
    __syncthreads();
    if (tok == a.eos) {
      stop = 0;
      break;
    }
  }
  if (lead) {
    if (gen_mode) {
      a.status[ST_NGEN] = gen;
      a.status[ST_STOP] = stop;
      a.status[ST_HITS] = hits;
      a.status[ST_TRIES] = tries;
    }
    a.status[ST_FORWARDS] += f;  // a resumed launch adds to its prefill launch's count
    const uint64_t t = globaltimer();
    a.status[ST_TEND] = (int32_t)(uint32_t)t;
    a.status[ST_TEND + 1] = (int32_t)(uint32_t)(t >> 32);
  }
}

// Shared memory the kernel needs for a model / mmax / grid.
size_t decode_smem_bytes(const ModelDev& md, int srows, int grid) {
  const int mmax = srows;
  int actw = std::max(std::max(md.D, md.QKV), md.FF);
  actw = std::max(actw, 3 * grid + 4);
  actw = (actw + 3) & ~3;
  const int hist_cap = md.kv_len + 64;
  size_t words = (size_t)mmax * md.D + (size_t)mmax * actw + kWarps * 68 + hist_cap + 16 + 16 + hist_cap + 64 + 32;
  words = (words + 1) & ~(size_t)1;
  words += 2 * kWarps * 4 + kWarps * 4 + 2 * kWarps * 16;
  return words * 4;
}

typedef void (*DecodeFn)(const RunArgs);

// Instantiations by words-per-lane of a D-long and an FF-long row (ceil(n / 256)); `multi` selects the
// general kernel (prefill chunks, verify forwards, speculation) over the single-token decode kernel.
DecodeFn pick_decode_kernel(int D, int FF, bool multi) {
  const int nd = (D / 8 + 31) / 32, nf = (FF / 8 + 31) / 32;
#define MLLM_PICK(A, B) \
  if (nd <= A && nf <= B) return multi ? decode_kernel<A, B, true> : nullptr;
#ifndef MLLM_FAST_BUILD
  MLLM_PICK(1, 2)
#endif
  MLLM_PICK(3, 6)
#ifndef MLLM_FAST_BUILD
  MLLM_PICK(3, 12)
  MLLM_PICK(4, 10)
  MLLM_PICK(4, 16)
#endif
#undef MLLM_PICK
  return nullptr;
}

}  // namespace mllm
