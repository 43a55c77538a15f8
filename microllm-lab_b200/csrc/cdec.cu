// Cluster decode kernel: the greedy single-token decode loop of engine/infer.js:625-639 (each token is
// forwardDecode, engine/infer.js:579-601) for llama-arch files, as ONE thread-block cluster of 16 CTAs
// (one per SM) that stays resident for every token of the call.
//
// Per layer, five stages; each ends with an all-to-all exchange through distributed shared memory:
// every CTA pushes its slice of the stage output into the same buffer of all 16 CTAs with st.async,
// and each receiving buffer has an mbarrier that completes when all of the stage's bytes have landed.
//
//   x (+ sum of squares)  -> QKV rows (x 1/RMS)                   -> qkv        (all CTAs)
//   qkv -> RoPE, causal attention of unit (kv head, position split) -> partials  (all CTAs)
//   partials -> merge -> proj rows + residual                      -> x1 (+ ss) (all CTAs)
//   x1 -> w1/w3 rows (x 1/RMS) -> SiLU(u) * v                      -> h         (all CTAs)
//   h -> w2 rows + residual                                         -> x2 (+ ss) (all CTAs)
// then the final RMSNorm, the lm_head rows of each CTA with a local argmax, and an exchange of the 16
// candidates (engine/infer.js:240-250: the lowest index wins a tie).
//
// Row dot products run on the tensor cores (mma.sync m16n8k16, fp32 accumulation): a 16-row x 32-wide
// weight group is one record of a warp's private stream; nibbles become exact fp16 (q - 8) with four
// LOP3 and four half2 fix-ups per 8 values; the activation is split into fp16 hi + lo halves that fill
// B columns 0 and 1 (relative residual <= 2^-22); each group's sum is scaled by its fp32 scale.  The
// weights are repacked at load time into one stream per (CTA, warp) in the order the warp consumes
// them, and every warp keeps a ring of kCdRing records filled ahead of use with 16-byte cp.async, so
// weight fetch from L2 overlaps the exchanges.  On one 16-SM cluster a 16-byte load stream reaches
// about 1.25 TB/s and an all-to-all exchange costs about 0.4 us (measured on B200).
//
// Every wait is bounded (RunArgs::wait_ns, default 0.5 s).  A CTA whose wait runs out raises the
// device error flag; the others see it in their next wait; all CTAs then meet at the final cluster
// barrier (so no CTA leaves while another may still write into its shared memory) and return.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "cdec.cuh"
#include "device_common.cuh"
#include "q4mma.cuh"

namespace mllm {
namespace cd {

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
  uint32_t o;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(o) : "r"(a), "r"(rank));
  return o;
}
// 16-byte store into CTA `rank`'s shared memory; completes bytes on that CTA's mbarrier.
__device__ __forceinline__ void st_async4(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void bar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
// One arrival plus the bytes the next phase waits for.
__device__ __forceinline__ void bar_arm(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void cp_async16_cg(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_upto(uint32_t pending) {
  switch (pending) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
  }
}
__device__ __forceinline__ float2 ldcg_f2(const float* p) {
  float2 v;
  asm volatile("ld.global.cg.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
  return v;
}

enum { B_X2 = 0, B_QKV = 1, B_ATT = 2, B_X1 = 3, B_H = 4, B_CAND = 5, B_COUNT = 6 };

// A warp's weight stream: records [0, n) per token, repeated every token; `iss` records have been
// requested (in groups of kCdBatch), `con` consumed.  Record r lives in ring slot r % kCdRing.
struct Ring {
  const uint4* src;
  uint8_t* buf;
  uint32_t n, iss, con;
};

// Request batches while the ring has room for one.
__device__ __forceinline__ void ring_issue(Ring& R, int lane) {
  while (R.iss - R.con + kCdBatch <= kCdRing) {
#pragma unroll
    for (int b = 0; b < kCdBatch; ++b) {
      const uint32_t rec = R.iss + b;
      if (lane < kCdRecBytes / 16)
        cp_async16_cg(R.buf + (rec % kCdRing) * kCdRecBytes + lane * 16, R.src + (size_t)(rec % R.n) * 20 + lane);
    }
    cp_commit();
    R.iss += kCdBatch;
  }
}

// Make record R.con readable by the whole warp (at the start of each batch: refill first, then wait
// for the batch's group).
__device__ __forceinline__ void ring_ready(Ring& R, int lane) {
  if (R.con % kCdBatch == 0) {
    __syncwarp();
    ring_issue(R, lane);
    cp_wait_upto(R.iss / kCdBatch - R.con / kCdBatch - 1);
    __syncwarp();
  }
}

// (q - 8) of the 8 nibbles of one word as 4 fp16 pairs: (k0,k4), (k1,k5), (k2,k6), (k3,k7), where
// byte j of the word holds k 2j (low nibble) and 2j + 1 (high).  Every step is exact in fp16.
__device__ __forceinline__ void dq8(uint32_t w, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  uint32_t q0 = (w & 0x000F000Fu) | 0x64006400u;
  uint32_t q1 = (w & 0x00F000F0u) | 0x64006400u;
  uint32_t q2 = (w8 & 0x000F000Fu) | 0x64006400u;
  uint32_t q3 = (w8 & 0x00F000F0u) | 0x64006400u;
  const __half2 off = __halves2half2(__float2half_rn(-1032.f), __float2half_rn(-1032.f));
  const __half2 s16 = __halves2half2(__float2half_rn(0.0625f), __float2half_rn(0.0625f));
  const __half2 off16 = __halves2half2(__float2half_rn(-72.f), __float2half_rn(-72.f));
  __half2 r0 = __hadd2(*reinterpret_cast<__half2*>(&q0), off);
  __half2 r1 = __hfma2(*reinterpret_cast<__half2*>(&q1), s16, off16);
  __half2 r2 = __hadd2(*reinterpret_cast<__half2*>(&q2), off);
  __half2 r3 = __hfma2(*reinterpret_cast<__half2*>(&q3), s16, off16);
  o[0] = *reinterpret_cast<uint32_t*>(&r0);
  o[1] = *reinterpret_cast<uint32_t*>(&r1);
  o[2] = *reinterpret_cast<uint32_t*>(&r2);
  o[3] = *reinterpret_cast<uint32_t*>(&r3);
}

// One record: rows gid / gid + 8 of the tile, this lane's k values 8t..8t+7 of the group.  A step-0
// fragment takes k (8t, 8t+4) and (8t+1, 8t+5), step 1 (8t+2, 8t+6) and (8t+3, 8t+7); the B fragments
// in `bf` follow the same order (build_bfrag).  Lanes with t == 0 accumulate rows gid and gid + 8.
__device__ __forceinline__ void unit_mma(const uint8_t* rec, const uint4* bf_g, int lane, float& acc0, float& acc1) {
  const int gid = lane >> 2, t = lane & 3;
  const uint2 wv = *reinterpret_cast<const uint2*>(rec + 8 * lane);
  const float2 sc = *reinterpret_cast<const float2*>(rec + 256 + 8 * gid);
  uint4 b = make_uint4(0u, 0u, 0u, 0u);
  if (gid < 2) b = bf_g[gid * 4 + t];
  uint32_t p[4], q[4];
  dq8(wv.x, p);
  dq8(wv.y, q);
  float c[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t a0[4] = {p[0], q[0], p[1], q[1]};
  const uint32_t a1[4] = {p[2], q[2], p[3], q[3]};
  mma16816(c, a0, b.x, b.y);
  mma16816(c, a1, b.z, b.w);
  acc0 = fmaf(c[0] + c[1], sc.x, acc0);
  acc1 = fmaf(c[2] + c[3], sc.y, acc1);
}

// B fragments of a K-long activation (times `gain` when given): bf[g][half][t] = 4 registers of fp16
// pairs (x[8t], x[8t+4]), (x[8t+1], x[8t+5]), (x[8t+2], x[8t+6]), (x[8t+3], x[8t+7]) of group g,
// half 0 = hi, 1 = lo.
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}
__device__ void build_bfrag(const float* x, const float* gain, int K, uint4* bf) {
  const int G = K >> 5;
  for (int q = threadIdx.x; q < G * 4; q += kCdThreads) {
    const int g = q >> 2, t = q & 3, k0 = 32 * g + 8 * t;
    __half hi[8], lo[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = gain ? x[k0 + j] * __ldg(gain + k0 + j) : x[k0 + j];
      split_hi_lo(v, hi[j], lo[j]);
    }
    bf[(g * 2) * 4 + t] = make_uint4(pack_h2(hi[0], hi[4]), pack_h2(hi[1], hi[5]), pack_h2(hi[2], hi[6]),
                                     pack_h2(hi[3], hi[7]));
    bf[(g * 2 + 1) * 4 + t] = make_uint4(pack_h2(lo[0], lo[4]), pack_h2(lo[1], lo[5]), pack_h2(lo[2], lo[6]),
                                         pack_h2(lo[3], lo[7]));
  }
}

// This warp's share of one stage: partial row sums per (unit tile, k slice) into red.
__device__ __forceinline__ void run_units(Ring& R, const CdGeom& g, const uint4* bf, float* red, int warp, int lane) {
  const int ks = warp % g.KW, ts = warp / g.KW;
  const int g0 = ks * g.G / g.KW, g1 = (ks + 1) * g.G / g.KW;
  for (int tl = ts; tl < g.Tu; tl += g.TW) {
    float a0 = 0.f, a1 = 0.f;
    for (int gg = g0; gg < g1; ++gg) {
      ring_ready(R, lane);
      unit_mma(R.buf + (R.con % kCdRing) * kCdRecBytes, bf + gg * 8, lane, a0, a1);
      ++R.con;
    }
    if ((lane & 3) == 0) {
      float* r = red + (tl * g.KW + ks) * 16 + (lane >> 2);
      r[0] = a0;
      r[8] = a1;
    }
  }
}

// Row i (0 .. 16 Tu) of the CTA's unit tiles: the k-slice partials summed in slice order.
__device__ __forceinline__ float row_sum(const float* red, const CdGeom& g, int i) {
  const float* r = red + (i >> 4) * g.KW * 16 + (i & 15);
  float s = 0.f;
  for (int k = 0; k < g.KW; ++k) s += r[k * 16];
  return s;
}

// Send n floats (n % 4 == 0) from this CTA's src to shared address `dst` (the same buffer in every
// CTA), completing on barrier `bar` of each CTA.
__device__ __forceinline__ void push_all(const float* src, uint32_t dst, int n, uint32_t bar) {
  const int n4 = n >> 2;
  for (int i = threadIdx.x; i < kCdCtas * n4; i += kCdThreads) {
    const int d = i / n4, q = i - d * n4;
    const float4 v = reinterpret_cast<const float4*>(src)[q];
    st_async4(mapa(dst + 16 * q, d), v, mapa(bar, d));
  }
}

// Bounded wait of the whole CTA for `parity` of a local barrier; false everywhere when it gave up.
__device__ __forceinline__ bool xwait(uint32_t bar, uint32_t parity, int* err, uint64_t limit) {
  bool ok = true;
  if (!bar_try(bar, parity)) {
    const uint64_t t0 = globaltimer();
    int n = 0;
    while (!bar_try(bar, parity)) {
      if ((++n & 15) == 0 && (*(volatile int*)err || globaltimer() - t0 > limit)) {
        atomicCAS(err, 0, 1);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok);
}

// Sum of squares of this CTA's n values v (held by threads 0..n-1), in a fixed order; result in misc[16].
__device__ __forceinline__ void block_ss(float v, float* misc) {
  float s = warp_sum(v * v);
  if ((threadIdx.x & 31) == 0) misc[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kCdWarps; ++w) t += misc[w];
    misc[16] = t;
  }
  __syncthreads();
}

__device__ __forceinline__ float inv_rms(const float* xb, int D) {
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kCdCtas; ++c) s += xb[D + 4 * c];
  return 1.f / sqrtf(s / D + 1e-6f);
}

}  // namespace cd

using namespace cd;

__global__ void __launch_bounds__(kCdThreads, 1) cdec_kernel(const __grid_constant__ CdArgs A) {
  extern __shared__ __align__(16) uint8_t smem[];
  const RunArgs& a = A.r;
  const ModelDev& md = a.m;
  const CdSmem Ls = cd_smem(md);
  const int c = (int)cta_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = md.D, QKV = md.QKV, FF = md.FF, NKV = md.NKV, rep = md.NH / md.NKV;
  const int S = cd_splits(md), U = NKV * S;
  uint4* bfrag = reinterpret_cast<uint4*>(smem + Ls.bfrag);
  float* red = reinterpret_cast<float*>(smem + Ls.red);
  float* xb2 = reinterpret_cast<float*>(smem + Ls.xb2);
  float* xb1 = reinterpret_cast<float*>(smem + Ls.xb1);
  float* qkvb = reinterpret_cast<float*>(smem + Ls.qkv);
  float* hb = reinterpret_cast<float*>(smem + Ls.hb);
  float* attb = reinterpret_cast<float*>(smem + Ls.attb);
  float* cand = reinterpret_cast<float*>(smem + Ls.cand);
  float* att = reinterpret_cast<float*>(smem + Ls.att);
  float* outv = reinterpret_cast<float*>(smem + Ls.outv);
  float* wpart = reinterpret_cast<float*>(smem + Ls.wpart);
  float* qk = reinterpret_cast<float*>(smem + Ls.qk);
  float* misc = reinterpret_cast<float*>(smem + Ls.misc);
  int* imisc = reinterpret_cast<int*>(misc);
  const uint32_t sbar = smem_u32(smem + Ls.bars);
  const uint32_t bytes_x = (uint32_t)(D * 4 + kCdCtas * 16);
  const uint32_t bar_bytes[B_COUNT] = {bytes_x, (uint32_t)QKV * 4, (uint32_t)(U * rep * kCdPartWords * 4), bytes_x,
                                       (uint32_t)FF * 4, (uint32_t)(kCdCtas * 16)};
  const uint64_t limit = a.wait_ns ? a.wait_ns : kWaitNs;
  uint32_t par[B_COUNT] = {0, 0, 0, 0, 0, 0};
  if (tid == 0) {
    for (int b = 0; b < B_COUNT; ++b) bar_init(sbar + 8 * b, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int b = 0; b < B_COUNT; ++b) bar_arm(sbar + 8 * b, bar_bytes[b]);
  }
  __syncthreads();
  cluster_sync_all();  // every barrier is armed before any CTA sends

  // bounded wait + re-arm for the next use of the same buffer
  auto wait_bar = [&](int b) -> bool {
    if (!xwait(sbar + 8 * b, par[b] & 1, a.err, limit)) return false;
    ++par[b];
    if (tid == 0) bar_arm(sbar + 8 * b, bar_bytes[b]);
    return true;
  };

  Ring R;
  R.src = A.wst + (size_t)A.woff[c * kCdWarps + warp] * (kCdRecBytes / 16);
  R.buf = smem + Ls.ring + warp * kCdRing * kCdRecBytes;
  R.n = A.wcnt[c * kCdWarps + warp];
  R.iss = R.con = 0;

  const bool gen_mode = a.mode == MODE_GENERATE;
  int gen = 0, tok = 0, stop = 1, f = 0;
  bool ok = true;
  CdGeom gq, gp, gw13, gw2, glm;
  {
    int rows, K;
    bool pr;
    cd_stage_shape(md, CD_QKV, &rows, &K, &pr);
    gq = cd_geom(rows, K, pr, c);
    cd_stage_shape(md, CD_PROJ, &rows, &K, &pr);
    gp = cd_geom(rows, K, pr, c);
    cd_stage_shape(md, CD_W13, &rows, &K, &pr);
    gw13 = cd_geom(rows, K, pr, c);
    cd_stage_shape(md, CD_W2, &rows, &K, &pr);
    gw2 = cd_geom(rows, K, pr, c);
    cd_stage_shape(md, CD_LM, &rows, &K, &pr);
    glm = cd_geom(rows, K, pr, c);
  }
  if (a.mode == MODE_SELFTEST_WAIT) {
    // Failure-detection self-test: phase 0 of the candidate barrier needs bytes nobody sends; the
    // wait runs out its limit and raises the error flag.
    ok = xwait(sbar + 8 * B_CAND, 0, a.err, limit);
    goto done;
  }
  if (!gen_mode && a.mode != MODE_FORWARD) goto done;
  if (gen_mode) {
    if (*(volatile int*)a.err) goto done;
    gen = a.start_gen;
    tok = a.out_ids[gen - 1];
    if (tok == a.eos) stop = 0;
  }
  if (R.n) ring_issue(R, lane);

  for (;;) {
    int pos;
    if (gen_mode) {
      if (stop == 0 || gen >= a.max_new || a.n_ids + gen >= md.kv_len) break;  // engine/infer.js:625-628
      pos = a.n_ids + gen - 1;
    } else {
      if (f == 1) break;
      tok = a.ids[0];
      pos = a.pos0;
    }
    // ---- embed (engine/infer.js:360-420): the dequantised tied lm_head row, in every CTA
    {
      const uint8_t* row = reinterpret_cast<const uint8_t*>(md.lm.w) + (size_t)tok * (D / 2);
      const float* sc = md.lm.s + (size_t)tok * (D / 32);
      float ss = 0.f;
      for (int k = tid; k < D; k += kCdThreads) {
        const int b = row[k >> 1];
        const float v = (float)(((k & 1) ? (b >> 4) : (b & 15)) - 8) * sc[k >> 5];
        xb2[k] = v;
        ss = fmaf(v, v, ss);
      }
      ss = warp_sum(ss);
      if (lane == 0) misc[warp] = ss;
      __syncthreads();
      if (tid < 4 * kCdCtas) {
        float t = 0.f;
        if (tid == 0)
          for (int w = 0; w < kCdWarps; ++w) t += misc[w];
        xb2[D + tid] = t;  // slot 0 holds the whole sum, slots 1..15 zero
      }
      __syncthreads();
    }
    for (int l = 0; l < md.n_layers; ++l) {
      const LayerDev& Ly = md.layers[l];
      if (l > 0 && !(ok = wait_bar(B_X2))) goto done;
      const float inv1 = inv_rms(xb2, D);
      build_bfrag(xb2, Ly.norm1, D, bfrag);
      // attention unit of this CTA and the K/V rows its warp walks first (issued before the stage)
      const bool has_unit = c < U;
      const int kvh = c / S, sp = c % S;
      const int span = (pos + S) / S;
      const int p_lo = sp * span, p_hi = min(pos + 1, p_lo + span);
      const size_t kv_base = ((size_t)l * NKV + kvh) * md.kv_len;
      float2 kpre[kCdKvPre], vpre[kCdKvPre];
#pragma unroll
      for (int j = 0; j < kCdKvPre; ++j) {
        const int p = p_lo + warp + kCdWarps * j;
        if (has_unit && p < p_hi && p < pos) {
          kpre[j] = ldcg_f2(a.kc + (kv_base + p) * 64 + 2 * lane);
          vpre[j] = ldcg_f2(a.vc + (kv_base + p) * 64 + 2 * lane);
        } else {
          kpre[j] = vpre[j] = make_float2(0.f, 0.f);
        }
      }
      __syncthreads();
      // ---- QKV rows
      run_units(R, gq, bfrag, red, warp, lane);
      __syncthreads();
      for (int i = tid; i < gq.T * 16; i += kCdThreads) outv[i] = inv1 * row_sum(red, gq, i);
      __syncthreads();
      push_all(outv, smem_u32(qkvb + 16 * gq.t0), gq.T * 16, sbar + 8 * B_QKV);
      if (!(ok = wait_bar(B_QKV))) goto done;
      // ---- attention of unit (kvh, sp): RoPE'd q heads, new k and v into qk (engine/infer.js:442-495)
      if (has_unit) {
        const float* cs = md.rope_cos + (size_t)pos * md.rope_dim;
        const float* sn = md.rope_sin + (size_t)pos * md.rope_dim;
        const int rd = md.rope_dim, half = rd / 2;
        for (int i = tid; i < (rep + 2) * 64; i += kCdThreads) {
          const int vec = i >> 6, d = i & 63;
          const float* src = vec < rep ? qkvb + (kvh * rep + vec) * 64
                                       : vec == rep ? qkvb + D + kvh * 64 : qkvb + D + NKV * 64 + kvh * 64;
          float v = src[d];
          if (vec <= rep && d < rd) {
            if (d < half) v = fmaf(-src[d + half], sn[d], src[d] * cs[d]);
            else v = fmaf(src[d - half], sn[d], src[d] * cs[d]);
          }
          qk[i] = v;
        }
        __syncthreads();
        if (pos >= p_lo && pos < p_hi && tid < 128) {  // the cache row of this position (engine/infer.js:457-464)
          const int d = tid & 63;
          if (tid < 64) a.kc[(kv_base + pos) * 64 + d] = qk[rep * 64 + d];
          else a.vc[(kv_base + pos) * 64 + d] = qk[(rep + 1) * 64 + d];
          __threadfence();
        }
        float qr[4][2], m[4], lsum[4], o[4][2];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          qr[h][0] = h < rep ? qk[h * 64 + 2 * lane] : 0.f;
          qr[h][1] = h < rep ? qk[h * 64 + 2 * lane + 1] : 0.f;
          m[h] = -INFINITY;
          lsum[h] = 0.f;
          o[h][0] = o[h][1] = 0.f;
        }
        for (int j = 0;; ++j) {
          const int p = p_lo + warp + kCdWarps * j;
          if (p >= p_hi) break;
          float2 kk, vv;
          if (p == pos) {
            kk = make_float2(qk[rep * 64 + 2 * lane], qk[rep * 64 + 2 * lane + 1]);
            vv = make_float2(qk[(rep + 1) * 64 + 2 * lane], qk[(rep + 1) * 64 + 2 * lane + 1]);
          } else if (j < kCdKvPre) {
            kk = kpre[0];
            vv = vpre[0];
          } else {
            kk = ldcg_f2(a.kc + (kv_base + p) * 64 + 2 * lane);
            vv = ldcg_f2(a.vc + (kv_base + p) * 64 + 2 * lane);
          }
          // rotate the prefetched registers so that kpre[0] always belongs to the next position
#pragma unroll
          for (int q = 0; q + 1 < kCdKvPre; ++q) {
            kpre[q] = kpre[q + 1];
            vpre[q] = vpre[q + 1];
          }
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            if (h >= rep) break;
            const float sdot = warp_sum(fmaf(qr[h][1], kk.y, qr[h][0] * kk.x)) * 0.125f;  // 1/sqrt(64)
            const float nm = fmaxf(m[h], sdot);
            const float corr = m[h] == -INFINITY ? 0.f : expf(m[h] - nm);
            const float e = expf(sdot - nm);
            lsum[h] = fmaf(lsum[h], corr, e);
            o[h][0] = fmaf(e, vv.x, o[h][0] * corr);
            o[h][1] = fmaf(e, vv.y, o[h][1] * corr);
            m[h] = nm;
          }
        }
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (h >= rep) break;
          float* wp = wpart + (warp * rep + h) * kCdPartWords;
          if (lane == 0) {
            wp[0] = m[h];
            wp[1] = lsum[h];
          }
          wp[4 + 2 * lane] = o[h][0];
          wp[5 + 2 * lane] = o[h][1];
        }
        __syncthreads();
        // the CTA's partial per head: max, sum, 2 zero words, 64 unnormalised outputs
        for (int i = tid; i < rep * 64; i += kCdThreads) {
          const int h = i >> 6, d = i & 63;
          float M = -INFINITY;
          for (int w = 0; w < kCdWarps; ++w) {
            const float* wp = wpart + (w * rep + h) * kCdPartWords;
            if (wp[1] > 0.f) M = fmaxf(M, wp[0]);
          }
          float Lsum = 0.f, O = 0.f;
          for (int w = 0; w < kCdWarps; ++w) {
            const float* wp = wpart + (w * rep + h) * kCdPartWords;
            if (wp[1] > 0.f) {
              const float fct = expf(wp[0] - M);
              Lsum = fmaf(wp[1], fct, Lsum);
              O = fmaf(wp[4 + d], fct, O);
            }
          }
          float* op = outv + h * kCdPartWords;
          op[4 + d] = O;
          if (d == 0) {
            op[0] = M;
            op[1] = Lsum;
            op[2] = 0.f;
            op[3] = 0.f;
          }
        }
        __syncthreads();
        push_all(outv, smem_u32(attb + c * rep * kCdPartWords), rep * kCdPartWords, sbar + 8 * B_ATT);
      }
      if (!(ok = wait_bar(B_ATT))) goto done;
      // ---- merge the splits of every head, then proj rows + residual (x1)
      for (int i = tid; i < D; i += kCdThreads) {
        const int h = i >> 6, d = i & 63, kv = h / rep, j = h % rep;
        float M = -INFINITY;
        for (int s = 0; s < S; ++s) {
          const float* pp = attb + ((kv * S + s) * rep + j) * kCdPartWords;
          if (pp[1] > 0.f) M = fmaxf(M, pp[0]);
        }
        float Lsum = 0.f, O = 0.f;
        for (int s = 0; s < S; ++s) {
          const float* pp = attb + ((kv * S + s) * rep + j) * kCdPartWords;
          if (pp[1] > 0.f) {
            const float fct = expf(pp[0] - M);
            Lsum = fmaf(pp[1], fct, Lsum);
            O = fmaf(pp[4 + d], fct, O);
          }
        }
        att[i] = O / Lsum;
      }
      __syncthreads();
      build_bfrag(att, nullptr, D, bfrag);
      __syncthreads();
      run_units(R, gp, bfrag, red, warp, lane);
      __syncthreads();
      {
        float v = 0.f;
        if (tid < gp.T * 16) {
          v = xb2[16 * gp.t0 + tid] + row_sum(red, gp, tid);
          outv[tid] = v;
        }
        block_ss(v, misc);  // needs gp.T * 16 <= kCdThreads
      }
      push_all(outv, smem_u32(xb1 + 16 * gp.t0), gp.T * 16, sbar + 8 * B_X1);
      if (tid < kCdCtas)
        st_async4(mapa(smem_u32(xb1 + D + 4 * c), tid), make_float4(misc[16], 0.f, 0.f, 0.f), mapa(sbar + 8 * B_X1, tid));
      if (!(ok = wait_bar(B_X1))) goto done;
      // ---- w1 / w3 rows, SiLU(u) * v (engine/infer.js:506-527)
      const float inv2 = inv_rms(xb1, D);
      build_bfrag(xb1, Ly.norm2, D, bfrag);
      __syncthreads();
      run_units(R, gw13, bfrag, red, warp, lane);
      __syncthreads();
      for (int i = tid; i < gw13.T * 16; i += kCdThreads) {
        const int tl = i >> 4, r = i & 15;
        const float u = inv2 * row_sum(red, gw13, (2 * tl) * 16 + r);
        const float v = inv2 * row_sum(red, gw13, (2 * tl + 1) * 16 + r);
        outv[i] = (u / (1.f + expf(-u))) * v;
      }
      __syncthreads();
      push_all(outv, smem_u32(hb + 16 * gw13.t0), gw13.T * 16, sbar + 8 * B_H);
      if (!(ok = wait_bar(B_H))) goto done;
      // ---- w2 rows + residual (x2)
      build_bfrag(hb, nullptr, FF, bfrag);
      __syncthreads();
      run_units(R, gw2, bfrag, red, warp, lane);
      __syncthreads();
      {
        float v = 0.f;
        if (tid < gw2.T * 16) {
          v = xb1[16 * gw2.t0 + tid] + row_sum(red, gw2, tid);
          outv[tid] = v;
        }
        block_ss(v, misc);
      }
      push_all(outv, smem_u32(xb2 + 16 * gw2.t0), gw2.T * 16, sbar + 8 * B_X2);
      if (tid < kCdCtas)
        st_async4(mapa(smem_u32(xb2 + D + 4 * c), tid), make_float4(misc[16], 0.f, 0.f, 0.f), mapa(sbar + 8 * B_X2, tid));
    }
    // ---- final RMSNorm, lm_head rows of this CTA, argmax candidates (engine/infer.js:240-250)
    if (!(ok = wait_bar(B_X2))) goto done;
    {
      const float invf = inv_rms(xb2, D);
      build_bfrag(xb2, md.norm_f, D, bfrag);
      __syncthreads();
      run_units(R, glm, bfrag, red, warp, lane);
      __syncthreads();
      float best = -INFINITY;
      int bidx = 0x7fffffff;
      const int r0 = 16 * glm.t0;
      for (int i = tid; i < glm.T * 16; i += kCdThreads) {
        const int r = r0 + i;
        if (r >= md.vocab) break;
        const float v = invf * row_sum(red, glm, i);
        if (!gen_mode && a.logits) a.logits[r] = v;
        if (v > best) {  // rows rise per thread: strict > keeps the lowest index on ties
          best = v;
          bidx = r;
        }
      }
#pragma unroll
      for (int o2 = 16; o2 > 0; o2 >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o2);
        const int oi = __shfl_xor_sync(0xffffffffu, bidx, o2);
        if (ov > best || (ov == best && oi < bidx)) {
          best = ov;
          bidx = oi;
        }
      }
      if (lane == 0) {
        misc[32 + warp] = best;
        imisc[48 + warp] = bidx;
      }
      __syncthreads();
      if (tid < kCdCtas) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kCdWarps; ++w) {
          const float v = misc[32 + w];
          const int id = imisc[48 + w];
          if (v > bv || (v == bv && id < bi)) {
            bv = v;
            bi = id;
          }
        }
        st_async4(mapa(smem_u32(cand + 4 * c), tid), make_float4(bv, __int_as_float(bi), 0.f, 0.f),
                  mapa(sbar + 8 * B_CAND, tid));
      }
      if (!(ok = wait_bar(B_CAND))) goto done;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int cc = 0; cc < kCdCtas; ++cc) {
        const float v = cand[4 * cc];
        const int id = __float_as_int(cand[4 * cc + 1]);
        if (v > bv || (v == bv && id < bi)) {
          bv = v;
          bi = id;
        }
      }
      tok = bi;
    }
    ++f;
    if (!gen_mode) {
      if (c == 0 && tid == 0 && a.argmax_out) a.argmax_out[0] = tok;
      continue;
    }
    if (c == 0 && tid == 0) a.out_ids[gen] = tok;
    ++gen;
    if (tok == a.eos) stop = 0;
  }
done:
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (c == 0 && tid == 0 && a.mode != MODE_SELFTEST_WAIT && ok) {
    if (gen_mode) {
      a.status[ST_NGEN] = gen;
      a.status[ST_STOP] = stop;
    }
    a.status[ST_FORWARDS] += f;
    const uint64_t t = globaltimer();
    a.status[ST_TEND] = (int32_t)(uint32_t)t;
    a.status[ST_TEND + 1] = (int32_t)(uint32_t)(t >> 32);
  }
  __syncthreads();
  cluster_sync_all();
}

// ---------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------

// Whether the cluster kernel runs this model: llama arch, head_dim 64, at most 4 query heads per kv
// head, every exchanged vector a whole number of 16-row tiles, per-CTA stage rows within the thread
// count (the residual stages keep one row per thread), and the shared-memory plan within `smem_cap`.
bool cd_supported(const ModelDev& m, size_t smem_cap) {
  if (m.arch != 0 || m.D != m.NH * 64 || m.NH % m.NKV || m.NH / m.NKV > 4) return false;
  if (m.D % 16 || m.QKV % 16 || m.FF % 16 || m.D % 32 || m.FF % 32) return false;
  if (m.NKV > kCdCtas || m.rope_dim > 64 || m.rope_dim % 2) return false;
  for (int c = 0; c < kCdCtas; ++c) {
    if (cd_geom(m.D, m.D, false, c).T * 16 > kCdThreads) return false;
    if (cd_geom(m.D, m.FF, false, c).T * 16 > kCdThreads) return false;
  }
  return (size_t)cd_smem(m).total <= smem_cap;
}

size_t cd_smem_bytes(const ModelDev& m) { return (size_t)cd_smem(m).total; }

// Records of every (CTA, warp) stream, in consumption order: per layer QKV, PROJ, W13 (w1 / w3 tiles
// interleaved), W2, then the lm_head.  A record holds, for lane = 4 gid + t, the words t of group g of
// rows gid and gid + 8 (8 bytes at 8 lane), then the scales of rows (gid, gid + 8) as a float pair at
// 256 + 8 gid.  Rows past the end hold q = 8 nibbles and zero scales.
void cd_pack(const ModelDev& m, const std::vector<HostQ4>& mats /* per layer: qkv, proj, w1, w3, w2 */,
             const HostQ4& lm, std::vector<uint8_t>* out, std::vector<uint32_t>* off, std::vector<uint32_t>* cnt) {
  off->assign(kCdCtas * kCdWarps, 0);
  cnt->assign(kCdCtas * kCdWarps, 0);
  size_t total = 0;
  // count
  auto stage_units = [&](int st, int c, int w) {
    int rows, K;
    bool paired;
    cd_stage_shape(m, st, &rows, &K, &paired);
    const CdGeom g = cd_geom(rows, K, paired, c);
    const int ks = w % g.KW, ts = w / g.KW;
    const int ng = (ks + 1) * g.G / g.KW - ks * g.G / g.KW;
    const int nt = ts < g.Tu ? (g.Tu - ts + g.TW - 1) / g.TW : 0;
    return (size_t)nt * ng;
  };
  for (int c = 0; c < kCdCtas; ++c)
    for (int w = 0; w < kCdWarps; ++w) {
      size_t n = 0;
      for (int st = CD_QKV; st <= CD_W2; ++st) n += stage_units(st, c, w) * m.n_layers;
      n += stage_units(CD_LM, c, w);
      (*off)[c * kCdWarps + w] = (uint32_t)total;
      (*cnt)[c * kCdWarps + w] = (uint32_t)n;
      total += n;
    }
  out->assign(total * kCdRecBytes, 0);
  uint8_t* dst = out->data();
  auto emit = [&](const HostQ4& q, int r0, int g) {
    const int hb = q.K / 2, ng = q.K / 32;
    for (int lane = 0; lane < 32; ++lane) {
      const int gid = lane >> 2, t = lane & 3;
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + gid + 8 * h;
        uint32_t word = 0x88888888u;
        if (r < q.rows) memcpy(&word, q.w + (size_t)r * hb + 16 * g + 4 * t, 4);
        memcpy(dst + 8 * lane + 4 * h, &word, 4);
      }
    }
    for (int gid = 0; gid < 8; ++gid)
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + gid + 8 * h;
        float s = 0.f;
        if (r < q.rows) memcpy(&s, q.s + ((size_t)r * ng + g) * 4, 4);
        memcpy(dst + 256 + 8 * gid + 4 * h, &s, 4);
      }
    dst += kCdRecBytes;
  };
  auto emit_stage = [&](int st, int c, int w, const HostQ4* a, const HostQ4* b) {
    int rows, K;
    bool paired;
    cd_stage_shape(m, st, &rows, &K, &paired);
    const CdGeom g = cd_geom(rows, K, paired, c);
    const int ks = w % g.KW, ts = w / g.KW;
    const int g0 = ks * g.G / g.KW, g1 = (ks + 1) * g.G / g.KW;
    for (int tl = ts; tl < g.Tu; tl += g.TW) {
      const HostQ4& q = paired ? ((tl & 1) ? *b : *a) : *a;
      const int tile = g.t0 + (paired ? tl / 2 : tl);
      for (int gg = g0; gg < g1; ++gg) emit(q, 16 * tile, gg);
    }
  };
  for (int c = 0; c < kCdCtas; ++c)
    for (int w = 0; w < kCdWarps; ++w) {
      for (int l = 0; l < m.n_layers; ++l) {
        const HostQ4* L = &mats[(size_t)l * 5];
        emit_stage(CD_QKV, c, w, &L[0], nullptr);
        emit_stage(CD_PROJ, c, w, &L[1], nullptr);
        emit_stage(CD_W13, c, w, &L[2], &L[3]);
        emit_stage(CD_W2, c, w, &L[4], nullptr);
      }
      emit_stage(CD_LM, c, w, &lm, nullptr);
    }
}

// Kernel attributes (once per process): the cluster of 16 is a non-portable size.
cudaError_t cd_setup(size_t smem_cap) {
  cudaError_t e = cudaFuncSetAttribute((const void*)cdec_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute((const void*)cdec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_cap);
}

// Clusters of this shape the device can hold at once (0: the kernel cannot run).
int cd_max_clusters(size_t smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCdCtas);
  cfg.blockDim = dim3(kCdThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kCdCtas;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, (void*)cdec_kernel, &cfg) != cudaSuccess) return 0;
  return n;
}

cudaError_t cd_launch(const CdArgs& args, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCdCtas);
  cfg.blockDim = dim3(kCdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kCdCtas;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  void* params[] = {const_cast<CdArgs*>(&args)};
  return cudaLaunchKernelExC(&cfg, (const void*)cdec_kernel, params);
}

}  // namespace mllm
