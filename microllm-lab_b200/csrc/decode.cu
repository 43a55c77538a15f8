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
  __device__ __forceinline__ void load(const Q4& q, int row, int nwords, int lane) {
    const uint32_t* wr = q.w + (size_t)row * nwords;
    const float* sr = q.s + (size_t)row * (nwords >> 2);
#pragma unroll
    for (int j = 0; j < NWJ; ++j) {
      const int k = lane + 32 * j;
      if (k < nwords) {
        w[j] = __ldg(wr + k);
        s[j] = __ldg(sr + (k >> 2));
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
};

struct Ctx {
  const RunArgs& a;
  Smem sm;
  Waiter wt;
  int lane, warp, gw, NW, G, actw, hist_cap;
  __device__ Ctx(const RunArgs& args) : a(args) {}
};

__device__ __forceinline__ bool cta_has_rows(int rows) { return (int)blockIdx.x * kWarps < rows; }

// RMSNorm (engine/infer.js:134-143) or LayerNorm (engine/infer.js:147-164) of rows xs[rows_from + i]
// into act[i], i < count.  One warp per row; f64 statistics.
__device__ void norm_rows(Ctx& c, const float* g, int rows_from, int count) {
  const int D = c.a.m.D;
  for (int i = c.warp; i < count; i += kWarps) {
    const float* x = c.sm.xs + (size_t)(rows_from + i) * D;
    float* o = c.sm.act + (size_t)i * c.actw;
    if (c.a.m.arch == 0) {
      double ss = 0;
      for (int k = c.lane; k < D; k += 32) ss += (double)x[k] * x[k];
      ss = warp_sum_d(ss);
      const double inv = 1.0 / sqrt(ss / D + 1e-6);
      for (int k = c.lane; k < D; k += 32) o[k] = (float)((double)x[k] * inv * (double)g[k]);
    } else {
      double mean = 0;
      for (int k = c.lane; k < D; k += 32) mean += x[k];
      mean = warp_sum_d(mean) / D;
      double v = 0;
      for (int k = c.lane; k < D; k += 32) {
        const double del = x[k] - mean;
        v += del * del;
      }
      v = warp_sum_d(v);
      const double inv = 1.0 / sqrt(v / D + 1e-5);
      for (int k = c.lane; k < D; k += 32) o[k] = (float)((x[k] - mean) * inv * (double)g[k] + (double)g[D + k]);
    }
  }
  __syncthreads();
}

// Wait for `rows` x `cols` words whose row r starts at rowptr(r); values land in dst[r * dstride + j].
template <class RowPtr>
__device__ bool poll_gather(Ctx& c, RowPtr rowptr, float* dst, int dstride, int rows, int cols, uint32_t tag) {
  const int n = rows * cols;
  bool ok = true;
  for (int base = threadIdx.x; base < n && ok; base += kThreads * 8) {
    uint32_t pending = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
      if (base + k * kThreads < n) pending |= 1u << k;
    const uint64_t t0 = globaltimer();
    int rounds = 0;
    while (pending) {
      uint64_t v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (pending & (1u << k)) {
          const int i = base + k * kThreads;
          v[k] = ll_load(rowptr(i / cols) + (i % cols));
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if ((pending & (1u << k)) && (uint32_t)(v[k] >> 32) == tag) {
          const int i = base + k * kThreads;
          dst[(i / cols) * dstride + (i % cols)] = __uint_as_float((uint32_t)v[k]);
          pending &= ~(1u << k);
        }
      }
      if (pending && ((++rounds & 31) == 0) && c.wt.give_up(t0)) {
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

// GEMV over the rows this warp owns: out(r, i, value) for token rows i < M.  The first row's weights
// are loaded before `wait()` (which polls the stage input and may normalise it) so that their latency
// hides behind the wait.  Ends with a CTA barrier: the next stage may overwrite `x`.
template <int NWJ, class Wait, class Out>
__device__ bool gemv_stage(Ctx& c, const Q4& q, int R, int n, const float* x, int ld, int M, Wait wait, Out out) {
  const int nwords = n >> 3;
  RowW<NWJ> rw;
  int r = c.gw;
  if (r < R) rw.load(q, r, nwords, c.lane);
  if (!wait()) return false;
  for (; r < R; r += c.NW) {
    if (r != c.gw) rw.load(q, r, nwords, c.lane);
    if (M == 1) {
      float v[1];
      rw.template dot<1>(x, ld, 1, nwords, c.lane, v);
      out(r, 0, v[0]);
    } else {
      for (int m0 = 0; m0 < M; m0 += 4) {
        float v[4];
        rw.template dot<4>(x + (size_t)m0 * ld, ld, M - m0, nwords, c.lane, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) out(r, m0 + i, v[i]);
      }
    }
  }
  __syncthreads();
  return true;
}

// Two matrices sharing rows and input (w1 and w3): out(r, i, u, v).
template <int NWJ, class Wait, class Out>
__device__ bool gemv2_stage(Ctx& c, const Q4& q1, const Q4& q3, int R, int n, const float* x, int ld, int M, Wait wait,
                            Out out) {
  const int nwords = n >> 3;
  RowW<NWJ> r1, r3;
  int r = c.gw;
  if (r < R) {
    r1.load(q1, r, nwords, c.lane);
    r3.load(q3, r, nwords, c.lane);
  }
  if (!wait()) return false;
  for (; r < R; r += c.NW) {
    if (r != c.gw) {
      r1.load(q1, r, nwords, c.lane);
      r3.load(q3, r, nwords, c.lane);
    }
    if (M == 1) {
      float u[1], v[1];
      r1.template dot<1>(x, ld, 1, nwords, c.lane, u);
      r3.template dot<1>(x, ld, 1, nwords, c.lane, v);
      out(r, 0, u[0], v[0]);
    } else {
      for (int m0 = 0; m0 < M; m0 += 4) {
        float u[4], v[4];
        r1.template dot<4>(x + (size_t)m0 * ld, ld, M - m0, nwords, c.lane, u);
        r3.template dot<4>(x + (size_t)m0 * ld, ld, M - m0, nwords, c.lane, v);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) out(r, m0 + i, u[i], v[i]);
      }
    }
  }
  __syncthreads();
  return true;
}

// Causal attention of one (head, token row) unit (engine/infer.js:422-495 for one q row).
__device__ bool attention_unit(Ctx& c, int l, int h, int m, int pos0, uint32_t tag) {
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
  if (!poll_gather(c, rowptr, q, 64, 1 + 2 * nloc, 64, tag)) return false;
  // RoPE on q (position pos_m) and on local k rows (engine/infer.js:208-225), f64 then f32.
  if (md.arch == 0 && md.rope_dim > 0) {
    const int half = md.rope_dim / 2;
    for (int t = threadIdx.x; t < (1 + nloc) * half; t += kThreads) {
      const int row = t / half, d = t % half;
      float* v = row == 0 ? q : kl + (size_t)(row - 1) * 64;
      const int pos = row == 0 ? pos_m : pos0 + row - 1;
      const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
      const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
      const float a0 = v[d], a1 = v[d + half];
      v[d] = (float)((double)a0 * cs[d] + (double)(-a1) * sn[d]);
      v[d + half] = (float)((double)a1 * cs[d + half] + (double)a0 * sn[d + half]);
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
  const float scale = 0.125f;  // 1/sqrt(64), exact (engine/infer.js:466)
  float mrun = -INFINITY, lrun = 0.f, o0 = 0.f, o1 = 0.f;
  for (int ch = c.warp; ch * 32 < npos; ch += kWarps) {
    const int p = ch * 32 + c.lane;
    float s = -INFINITY;
    if (p < npos) {
      float dot = 0.f;
      if (p < pos0) {
        const float4* kp = reinterpret_cast<const float4*>(c.a.kc + (kv_base + p) * 64);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float4 kv = __ldcg(kp + j);
          dot = fmaf(q[4 * j], kv.x, dot);
          dot = fmaf(q[4 * j + 1], kv.y, dot);
          dot = fmaf(q[4 * j + 2], kv.z, dot);
          dot = fmaf(q[4 * j + 3], kv.w, dot);
        }
      } else {
        const float* kp = kl + (size_t)(p - pos0) * 64;
#pragma unroll 16
        for (int d = 0; d < 64; ++d) dot = fmaf(q[d], kp[d], dot);
      }
      s = dot * scale;
    }
    const float cmax = warp_max(s);
    const float newm = fmaxf(mrun, cmax);
    const float e = p < npos ? expf(s - newm) : 0.f;
    const float corr = mrun == -INFINITY ? 0.f : expf(mrun - newm);
    lrun = lrun * corr + warp_sum(e);
    o0 *= corr;
    o1 *= corr;
    const int nj = min(32, npos - ch * 32);
    for (int j = 0; j < nj; ++j) {
      const float pj = __shfl_sync(0xffffffffu, e, j);
      const int pp = ch * 32 + j;
      const float* vp = pp < pos0 ? nullptr : vl + (size_t)(pp - pos0) * 64;
      float v0, v1;
      if (pp < pos0) {
        const float* vg = c.a.vc + (kv_base + pp) * 64;
        v0 = __ldcg(vg + c.lane);
        v1 = __ldcg(vg + c.lane + 32);
      } else {
        v0 = vp[c.lane];
        v1 = vp[c.lane + 32];
      }
      o0 = fmaf(pj, v0, o0);
      o1 = fmaf(pj, v1, o1);
    }
    mrun = newm;
  }
  float* wp = c.sm.wpart + c.warp * 68;
  if (c.lane == 0) {
    wp[0] = mrun;
    wp[1] = lrun;
  }
  wp[4 + c.lane] = o0;
  wp[4 + 32 + c.lane] = o1;
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
        r0 = fmaf(pw[4 + c.lane], f, r0);
        r1 = fmaf(pw[36 + c.lane], f, r1);
      }
    }
    const float inv = 1.f / L;
    uint64_t* dst = x.att + ((size_t)l * c.a.mmax + m) * x.s_d + h * kHeadDim;
    ll_store(dst + c.lane, tag, r0 * inv);
    ll_store(dst + 32 + c.lane, tag, r1 * inv);
  }
  __syncthreads();
  return true;
}

// GELU tanh form (engine/infer.js:166-171), f64.
__device__ __forceinline__ float gelu_new(float vf) {
  const double v = vf;
  return (float)(0.5 * v * (1 + tanh(0.7978845608028654 * (v + 0.044715 * v * v * v))));
}

// One forward over c.sm.toks[0..M) at positions pos0..; returns false when a wait gave up.
// lm: LM_NONE / LM_LAST / LM_EACH.  gpt2_hist (GPT-2 generate): apply argmaxGpt2 penalties using
// the generated ids sm.hist[hist_from .. hist_from + n_past).
template <int NWJ_D, int NWJ_F>
__device__ bool forward(Ctx& c, int M, int pos0, int lm, uint32_t tag, int parity, bool gpt2_pen, int hist_from,
                        int n_past, float* logits_out) {
  const RunArgs& a = c.a;
  const ModelDev& md = a.m;
  const ExchangeDev& x = a.x;
  const int D = md.D, FF = md.FF, QKV = md.QKV, mmax = a.mmax, actw = c.actw;
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
      if (md.sf) v = (float)((double)v / (double)md.sf[k]);
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
    const uint64_t* x2_prev = l > 0 ? x.x2 + (size_t)(l - 1) * mmax * x.s_d : nullptr;
    // ---------------- QKV (waits for the previous layer's x2 when the CTA needs the residual stream)
    if (cta_has_rows(QKV)) {
      uint64_t* dst = x.qkv + (size_t)l * mmax * x.s_qkv;
      const float* bias = L.qkv_b;
      auto wait = [&] {
        if (x2_prev && !poll_rowsof(x2_prev, x.s_d, sm.xs, D, D)) return false;
        norm_rows(c, L.norm1, 0, M);
        return true;
      };
      if (!gemv_stage<NWJ_D>(c, L.qkv, QKV, D, sm.act, actw, M, wait, [&](int r, int i, float v) {
            if (c.lane == 0) ll_store(dst + (size_t)i * x.s_qkv + r, tag, bias ? v + bias[r] : v);
          }))
        return false;
    } else if (x2_prev && cta_has_rows(D)) {
      if (!poll_rowsof(x2_prev, x.s_d, sm.xs, D, D)) return false;
    }
    // ---------------- ATT
    for (int u = blockIdx.x; u < md.NH * M; u += c.G) {
      if (!attention_unit(c, l, u % md.NH, u / md.NH, pos0, tag)) return false;
    }
    // ---------------- PROJ + residual
    if (cta_has_rows(D)) {
      const uint64_t* src = x.att + (size_t)l * mmax * x.s_d;
      uint64_t* dst = x.x1 + (size_t)l * mmax * x.s_d;
      const float* bias = L.proj_b;
      auto wait = [&] { return poll_rowsof(src, x.s_d, sm.act, actw, D); };
      if (!gemv_stage<NWJ_D>(c, L.proj, D, D, sm.act, actw, M, wait, [&](int r, int i, float v) {
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
      auto wait = [&] {
        if (!poll_rowsof(x1_l, x.s_d, sm.xs, D, D)) return false;
        norm_rows(c, L.norm2, 0, M);
        return true;
      };
      bool ok;
      if (md.arch == 0) {
        ok = gemv2_stage<NWJ_D>(c, L.w1, L.w3, FF, D, sm.act, actw, M, wait, [&](int r, int i, float u, float v) {
          if (c.lane == 0) {
            const double ud = u;
            ll_store(dst + (size_t)i * x.s_ff + r, tag, (float)((ud / (1 + exp(-ud))) * (double)v));
          }
        });
      } else {
        const float* bias = L.fc_b;
        ok = gemv_stage<NWJ_D>(c, L.w1, FF, D, sm.act, actw, M, wait, [&](int r, int i, float v) {
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
      if (!gemv_stage<NWJ_F>(c, L.w2, D, FF, sm.act, actw, M, wait, [&](int r, int i, float v) {
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
  const int nlm = lm == LM_EACH ? M : 1;
  const int lm_from = lm == LM_EACH ? 0 : M - 1;
  if (lm != LM_NONE) {
    if (!poll_rowsof(x2_last, x.s_d, sm.xs, D, D)) return false;
    norm_rows(c, md.norm_f, lm_from, nlm);
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
          if (r < md.vocab) rw[g].load(md.lm, r, nwords, c.lane);
        }
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
        const int r = r0 + g * c.NW;
        if (r >= md.vocab) break;
        float v[4];
        if (nlm == 1) {
          float v1[1];
          rw[g].template dot<1>(sm.act, actw, 1, nwords, c.lane, v1);
          v[0] = v1[0];
        } else {
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
__device__ int lookup_draft(Ctx& c, const int* seq, int len, int k, int n, int* out) {
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

template <int NWJ_D, int NWJ_F>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const RunArgs a) {
  extern __shared__ __align__(16) float smem[];
  Ctx c(a);
  c.lane = threadIdx.x & 31;
  c.warp = threadIdx.x >> 5;
  c.G = gridDim.x;
  c.gw = blockIdx.x * kWarps + c.warp;
  c.NW = c.G * kWarps;
  c.wt.err = a.err;
  c.wt.limit_ns = a.wait_ns ? a.wait_ns : kWaitNs;
  const ModelDev& md = a.m;
  const int mmax = a.mmax;
  int actw = max(max(md.D, md.QKV), md.FF);
  actw = max(actw, 3 * c.G * 1 + 4);
  actw = (actw + 3) & ~3;
  c.actw = actw;
  c.hist_cap = md.kv_len + 64;
  {
    float* p = smem;
    c.sm.xs = p; p += (size_t)mmax * md.D;
    c.sm.act = p; p += (size_t)mmax * actw;
    c.sm.wpart = p; p += kWarps * 68;
    c.sm.hist = reinterpret_cast<int*>(p); p += c.hist_cap;
    c.sm.toks = reinterpret_cast<int*>(p); p += 16;
    c.sm.res = reinterpret_cast<int*>(p); p += 16;
    c.sm.pen = reinterpret_cast<int*>(p); p += c.hist_cap + 64;
    c.sm.misc = reinterpret_cast<int*>(p); p += 32;
    p = reinterpret_cast<float*>(((uintptr_t)p + 7) & ~(uintptr_t)7);
    c.sm.cval = reinterpret_cast<double*>(p); p += 2 * kWarps * 4;
    c.sm.cidx = reinterpret_cast<int*>(p); p += kWarps * 4;
  }
  const bool lead = blockIdx.x == 0 && threadIdx.x == 0;
  if (lead) {
    const uint64_t t = globaltimer();
    a.status[ST_T0] = (int32_t)(uint32_t)t;
    a.status[ST_T0 + 1] = (int32_t)(uint32_t)(t >> 32);
  }
  int f = 0;  // forwards run in this launch
  const int n = a.n_ids;

  if (a.mode == MODE_SELFTEST_WAIT) {
    // Failure-detection self-test: every CTA waits for a candidate word with a tag no CTA writes in
    // this launch.  The wait runs out its limit, raises the error flag and the kernel returns; the
    // host reports MLLM_ERR_TIMEOUT and the context stays usable.
    const uint64_t* w = a.x.cand + (size_t)blockIdx.x * mmax * 4;
    poll_gather(c, [&](int) { return w; }, c.sm.act, 1, 1, 1, a.base_tag);
    return;
  }
  if (a.mode == MODE_FORWARD) {
    for (int c0 = 0; c0 < n; c0 += mmax) {
      const int M = min(mmax, n - c0);
      for (int t = threadIdx.x; t < M; t += kThreads) c.sm.toks[t] = a.ids[c0 + t];
      __syncthreads();
      const bool last = c0 + M >= n;
      const int lm = a.logits_each ? LM_EACH : (last ? LM_LAST : LM_NONE);
      float* lg = a.logits ? a.logits + (size_t)(a.logits_each ? c0 : 0) * md.vocab : nullptr;
      if (!forward<NWJ_D, NWJ_F>(c, M, a.pos0 + c0, lm, a.base_tag + f, f & 1, false, 0, 0, lg)) return;
      ++f;
      if (lead && a.argmax_out) {
        if (a.logits_each)
          for (int i = 0; i < M; ++i) a.argmax_out[c0 + i] = c.sm.res[i];
        else if (last)
          a.argmax_out[0] = c.sm.res[0];
      }
    }
    if (lead) a.status[ST_FORWARDS] = f;
  } else {
    // ------------------------------------------------------------ generate
    int* hist = c.sm.hist;
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
    int hlen = n, gen = 0, stop = 1 /* max_new_tokens */, hits = 0, tries = 0;
    const bool gpt2 = md.arch == 1;
    // prefill (engine/infer.js:611, engine/webgpu.js:1178-1186)
    for (int c0 = 0; c0 < n; c0 += mmax) {
      const int M = min(mmax, n - c0);
      for (int t = threadIdx.x; t < M; t += kThreads) c.sm.toks[t] = hist[c0 + t];
      __syncthreads();
      const bool last = c0 + M >= n;
      if (!forward<NWJ_D, NWJ_F>(c, M, c0, last ? LM_LAST : LM_NONE, a.base_tag + f, f & 1, gpt2, n, 0, nullptr))
        return;
      ++f;
    }
    int tok = c.sm.res[0];
    int cache = n < md.kv_len - 1 ? n : md.kv_len - 1;
    if (lead) {
      a.out_ids[0] = tok;
      const uint64_t t = globaltimer();
      a.status[ST_TFIRST] = (int32_t)(uint32_t)t;
      a.status[ST_TFIRST + 1] = (int32_t)(uint32_t)(t >> 32);
    }
    hist[hlen++] = tok;
    gen = 1;
    if (tok == a.eos) {
      stop = 0;
    } else if (a.spec_k <= 0) {
      // engine/infer.js:625-639
      for (int i = 1; i < a.max_new; ++i) {
        if (n + gen >= md.kv_len) break;
        if (threadIdx.x == 0) c.sm.toks[0] = tok;
        __syncthreads();
        if (!forward<NWJ_D, NWJ_F>(c, 1, n + gen - 1, LM_LAST, a.base_tag + f, f & 1, gpt2, n, gen, nullptr)) return;
        ++f;
        tok = c.sm.res[0];
        if (lead) a.out_ids[gen] = tok;
        hist[hlen++] = tok;
        ++gen;
        __syncthreads();
        if (tok == a.eos) {
          stop = 0;
          break;
        }
      }
    } else {
      // engine/webgpu.js:1239-1270 with lookupDraft over prompt + accepted ids
      int* draft = c.sm.pen;  // reused: speculation is llama-only
      while (gen < a.max_new) {
        if (cache >= md.kv_len - 1) break;
        const int xtok = tok;
        const int pos = cache;
        int dl = lookup_draft(c, hist, hlen, min(a.spec_k, mmax - 1), a.ngram, draft);
        if (pos + dl > md.kv_len - 1) dl = md.kv_len - 1 - pos;
        ++tries;
        if (threadIdx.x == 0) {
          c.sm.toks[0] = xtok;
          for (int i = 0; i < dl; ++i) c.sm.toks[1 + i] = draft[i];
        }
        __syncthreads();
        if (!forward<NWJ_D, NWJ_F>(c, 1 + dl, pos, dl > 0 ? LM_EACH : LM_LAST, a.base_tag + f, f & 1, false, 0, 0,
                                   nullptr))
          return;
        ++f;
        int r0 = c.sm.res[0];
        if (lead) a.out_ids[gen] = r0;
        hist[hlen++] = r0;
        ++gen;
        cache = pos + 1;
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
            cache = pos + 2 + k;
            tok = nxt;
            if (nxt == a.eos) break;
          }
        }
        __syncthreads();
        if (tok == a.eos) break;
      }
      if (tok == a.eos) stop = 0;
    }
    if (lead) {
      a.status[ST_NGEN] = gen;
      a.status[ST_STOP] = stop;
      a.status[ST_HITS] = hits;
      a.status[ST_TRIES] = tries;
      a.status[ST_FORWARDS] = f;
    }
  }
  if (lead) {
    const uint64_t t = globaltimer();
    a.status[ST_TEND] = (int32_t)(uint32_t)t;
    a.status[ST_TEND + 1] = (int32_t)(uint32_t)(t >> 32);
  }
}

// Shared memory the kernel needs for a model / mmax / grid.
size_t decode_smem_bytes(const ModelDev& md, int mmax, int grid) {
  int actw = std::max(std::max(md.D, md.QKV), md.FF);
  actw = std::max(actw, 3 * grid + 4);
  actw = (actw + 3) & ~3;
  const int hist_cap = md.kv_len + 64;
  size_t words = (size_t)mmax * md.D + (size_t)mmax * actw + kWarps * 68 + hist_cap + 16 + 16 + hist_cap + 64 + 32;
  words = (words + 1) & ~(size_t)1;
  words += 2 * kWarps * 4 + kWarps * 4;
  return words * 4;
}

typedef void (*DecodeFn)(const RunArgs);

// Instantiations by words-per-lane of a D-long and an FF-long row (ceil(n / 256)).
DecodeFn pick_decode_kernel(int D, int FF) {
  const int nd = (D / 8 + 31) / 32, nf = (FF / 8 + 31) / 32;
  if (nd <= 1 && nf <= 2) return decode_kernel<1, 2>;
  if (nd <= 3 && nf <= 6) return decode_kernel<3, 6>;
  if (nd <= 3 && nf <= 12) return decode_kernel<3, 12>;
  if (nd <= 4 && nf <= 10) return decode_kernel<4, 10>;
  if (nd <= 4 && nf <= 16) return decode_kernel<4, 16>;
  return nullptr;
}

}  // namespace mllm
