// Cluster decode kernel: the greedy single-token decode loop of engine/infer.js:625-639 (each token is
// forwardDecode, engine/infer.js:579-601) for llama-arch files, as ONE thread-block cluster of 16 CTAs
// (one per SM) that stays resident for every token of the call.
//
// Per layer, five stages; each ends with an all-to-all exchange through distributed shared memory:
// every CTA pushes its slice of the stage output into the same buffer of all 16 CTAs with st.async,
// and each receiving buffer has an mbarrier that completes when all of the stage's bytes have landed.
//
//   x (+ sums of squares)  -> QKV rows (x 1/RMS)                    -> qkv        (all CTAs)
//   qkv -> RoPE, causal attention of unit (kv head, position split) -> partials  (all CTAs)
//   partials -> merge -> proj rows + residual                       -> x1 (+ ss) (all CTAs)
//   x1 -> w1/w3 rows (x 1/RMS) -> SiLU(u) * v                       -> h         (all CTAs)
//   h -> w2 rows + residual                                          -> x2 (+ ss) (all CTAs)
// then the final RMSNorm, the lm_head rows of each CTA with a local argmax, and an exchange of the 16
// candidates (engine/infer.js:240-250: the lowest index wins a tie).
//
// Row dot products run on the CUDA cores in fp32 (engine/infer.js:88-116 with f32 instead of f64
// sums).  A 16-row x 32-wide weight group is one 320-byte record of a warp's private stream: lane
// (gid, t) holds word t (8 nibbles) of rows gid and gid + 8, and its four lanes t = 0..3 add their
// partial sums at the end of a tile.  A nibble becomes an exact fp32 (q - 8) 16^e with one LOP3
// (2^23 + q 16^e from the mantissa bits, e = 0..4) and one packed subtraction; the activation is
// stored pre-scaled by 16^-e, so every product (q - 8) x is formed exactly and rounded once, as a
// plain fp32 multiply would.  Packed f32x2 adds and FMAs halve the floating-point instructions.
// (Measured on B200: legacy mma.sync tiles were bound by the tensor pipe, about 21 pipe cycles per
// m16n8k16 per SM, 4x slower than this.)
//
// The weights are repacked at load time into one stream per CTA, in the order its warps consume
// them, cut into 40 KB chunks (8 records per warp); a ring of up to 4 chunk slots is filled by one
// bulk copy per chunk (cp.async.bulk, completing on the slot's mbarrier), so weight fetch runs a
// layer ahead of the exchanges.  (Measured on B200 from one 16-SM cluster: bulk copies of 40-64 KB
// stream 60-70 GB/s per SM; per-warp 16-byte cp.async rings reached about 36 GB/s.)  Per-layer
// vectors (norm gains, the RoPE row of the position) are fetched into registers a layer or a token
// ahead.
//
// Every wait is bounded (RunArgs::wait_ns, default 0.5 s).  A CTA whose wait runs out raises the
// device error flag; the others see it in their next wait; all CTAs then meet at the final cluster
// barrier (so no CTA leaves while another may still write into its shared memory) and return.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "cdec.cuh"
#include "device_common.cuh"

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
// Stores into CTA `rank`'s shared memory that complete their bytes on that CTA's mbarrier.
__device__ __forceinline__ void st_async4(uint32_t raddr, float4 v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
               : "memory");
}
__device__ __forceinline__ void st_async1(uint32_t raddr, float v, uint32_t rbar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(raddr),
               "r"(__float_as_uint(v)), "r"(rbar)
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
__device__ __forceinline__ float2 ldcg_f2(const float* p) {
  float2 v;
  asm volatile("ld.global.cg.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
  return v;
}

// Packed fp32 pairs (f32x2 adds and FMAs on sm_100).
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 up2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Nibble i of a word (bits 4i, element k = i of the lane's 8) is taken at the scale 16^e(i) that leaves
// it inside a float mantissa without a shift: e = 0..4 for i = 0..4 and, after one shift by 12 bits,
// e = 2..4 for i = 5..7.
__host__ __device__ constexpr int cd_nib_exp(int i) { return i < 5 ? i : i - 3; }

// sum_i (q_i - 8) x_i for the 8 nibbles of w against the pre-scaled activations a[i] = x_i 16^-e(i).
__device__ __forceinline__ float dot8(uint32_t w, const float4& a0, const float4& a1) {
  const uint32_t w12 = w >> 12;
  const float f0 = __uint_as_float((w & 0x0000Fu) | 0x4B000000u);
  const float f1 = __uint_as_float((w & 0x000F0u) | 0x4B000000u);
  const float f2 = __uint_as_float((w & 0x00F00u) | 0x4B000000u);
  const float f3 = __uint_as_float((w & 0x0F000u) | 0x4B000000u);
  const float f4 = __uint_as_float((w & 0xF0000u) | 0x4B000000u);
  const float f5 = __uint_as_float((w12 & 0x00F00u) | 0x4B000000u);
  const float f6 = __uint_as_float((w12 & 0x0F000u) | 0x4B000000u);
  const float f7 = __uint_as_float((w12 & 0xF0000u) | 0x4B000000u);
  // 2^23 + 8 * 16^e: subtracting it leaves (q - 8) 16^e exactly
  const uint64_t d01 = add2(pk2(f0, f1), pk2(-8388616.f, -8388736.f));
  const uint64_t d23 = add2(pk2(f2, f3), pk2(-8390656.f, -8421376.f));
  const uint64_t d45 = add2(pk2(f4, f5), pk2(-8912896.f, -8390656.f));
  const uint64_t d67 = add2(pk2(f6, f7), pk2(-8421376.f, -8912896.f));
  uint64_t p = mul2(d01, pk2(a0.x, a0.y));
  p = fma2(d23, pk2(a0.z, a0.w), p);
  p = fma2(d45, pk2(a1.x, a1.y), p);
  p = fma2(d67, pk2(a1.z, a1.w), p);
  const float2 r = up2(p);
  return r.x + r.y;
}

enum { B_X2 = 0, B_QKV = 1, B_ATT = 2, B_X1 = 3, B_H = 4, B_CAND = 5, B_COUNT = 6 };

// The CTA's weight ring: nslot chunk slots, each filled by one bulk copy that completes on the slot's
// full barrier.  Every warp waits for a chunk before its first record in it and releases the chunk
// after its last; the warp whose release completes the count of 16 issues the chunk nslot further on
// into the same slot, so no thread ever blocks on the producer side.  Chunk k of the kernel is chunk
// k % cpt of the CTA's per-token stream (the stream repeats every token).  A warp walks its records
// with an incremental pointer; chunk indices, slots and barrier phases advance once per chunk.
struct Feed {
  const uint8_t* src;   // this CTA's cpt chunks
  uint8_t* ring;        // nslot slots
  int* cnt;             // [nslot] releases of the slot's current chunk; [kCdMaxSlots + s] last chunk issued
  uint32_t full;        // shared address of the slot 0 full barrier (8 bytes per slot)
  uint32_t cpt, nslot;
  // this warp
  const uint8_t* cur;   // its next record
  uint32_t kc;          // global index of the chunk holding it
  uint32_t slot, phase; // kc % nslot and the parity of kc / nslot
  uint32_t ri;          // records of this warp already taken from chunk kc
  uint32_t tok_end;     // first chunk of the next token
};

__device__ __forceinline__ void feed_issue(Feed& F, uint32_t k) {
  const uint32_t s = k % F.nslot;
  F.cnt[kCdMaxSlots + s] = (int)k;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // earlier reads of the slot come first
  bar_arm(F.full + 8 * s, kCdChunk);
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(F.ring + (size_t)s * kCdChunk)),
               "l"(F.src + (size_t)(k % F.cpt) * kCdChunk), "r"((uint32_t)kCdChunk), "r"(F.full + 8 * s)
               : "memory");
}

__device__ __forceinline__ bool bar_try_cta(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait of one warp for the bytes of its current chunk.
__device__ __forceinline__ bool feed_wait(const Feed& F, int* err, uint64_t limit) {
  const uint32_t bar = F.full + 8 * F.slot;
  if (bar_try_cta(bar, F.phase)) return true;
  const uint64_t t0 = globaltimer();
  for (int n = 0;; ++n) {
    if (bar_try_cta(bar, F.phase)) return true;
    if ((n & 15) == 15 && (*(volatile int*)err || globaltimer() - t0 > limit)) {
      atomicCAS(err, 0, 1);
      return false;
    }
  }
}

// Release chunk kc (this warp is done with it) and move to the next one.
__device__ __forceinline__ void feed_next_chunk(Feed& F, int warp, int lane) {
  __syncwarp();
  if (lane == 0) {
    __threadfence_block();
    if (atomicAdd(&F.cnt[F.slot], 1) == kCdWarps - 1) {
      F.cnt[F.slot] = 0;
      feed_issue(F, F.kc + F.nslot);
    }
  }
  __syncwarp();
  ++F.kc;
  F.ri = 0;
  if (++F.slot == F.nslot) {
    F.slot = 0;
    F.phase ^= 1u;
  }
  F.cur = F.ring + (size_t)F.slot * kCdChunk + (size_t)warp * kCdRpc * kCdRecBytes;
}

// End of a token: release the chunk this warp left part-way and every later chunk of the token.
__device__ __forceinline__ bool feed_token_end(Feed& F, int warp, int lane, int* err, uint64_t limit) {
  if (F.ri) feed_next_chunk(F, warp, lane);
  while (F.kc < F.tok_end) {
    if (!feed_wait(F, err, limit)) return false;
    feed_next_chunk(F, warp, lane);
  }
  F.tok_end += F.cpt;
  return true;
}

// This warp's share of one stage (see CdGeom): its contiguous range of units; per tile the rows'
// partial sums over the range's groups, scaled per group, reduced over the lane quad, into
// red[(tile * maxc + slot) * 16 + row] (slot = this warp's order among the tile's warps).  False when a
// wait for weights gave up.
__device__ __forceinline__ bool run_units(Feed& F, const CdGeom& g, int off, const float* actp, float* red, int warp,
                                          int lane, int* err, uint64_t limit) {
  const int v = (warp - off) & (kCdWarps - 1);
  const int u1 = cd_ustart(g, v + 1);
  const int gid = lane >> 2, t = lane & 3;
  int u = cd_ustart(g, v);
  while (u < u1) {
    const int tl = u / g.G;
    const int ue = min(u1, (tl + 1) * g.G);
    const int slot = v - cd_vwarp(g, tl * g.G);
    const float* ap = actp + 32 * (u - tl * g.G) + 8 * t;
    float acc0 = 0.f, acc1 = 0.f;
    for (; u < ue; ++u, ap += 32) {
      if (F.ri == 0 && !feed_wait(F, err, limit)) return false;
      const uint2 wv = *reinterpret_cast<const uint2*>(F.cur + 8 * lane);
      const float2 sc = *reinterpret_cast<const float2*>(F.cur + 256 + 8 * gid);
      const float4 a0 = reinterpret_cast<const float4*>(ap)[0];
      const float4 a1 = reinterpret_cast<const float4*>(ap)[1];
      acc0 = fmaf(dot8(wv.x, a0, a1), sc.x, acc0);
      acc1 = fmaf(dot8(wv.y, a0, a1), sc.y, acc1);
      F.cur += kCdRecBytes;
      if (++F.ri == kCdRpc) feed_next_chunk(F, warp, lane);
    }
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    if (t == 0) {
      float* r = red + (tl * g.maxc + slot) * 16 + gid;
      r[0] = acc0;
      r[8] = acc1;
    }
  }
  return true;
}

// Row i (0 .. 16 Tu) of the CTA's unit tiles: the partials of the tile's warps, in warp order.
__device__ __forceinline__ float row_sum(const float* red, const CdGeom& g, int i) {
  const int tl = i >> 4;
  const int nc = cd_vwarp(g, tl * g.G + g.G - 1) - cd_vwarp(g, tl * g.G) + 1;
  const float* r = red + tl * g.maxc * 16 + (i & 15);
  float s = 0.f;
  for (int k = 0; k < nc; ++k) s += r[k * 16];
  return s;
}

// Pre-scaled stage activation for element k: x * 16^-e(k % 8) (exact).
__device__ __forceinline__ float pre_scale(float x, int k) {
  const int e = cd_nib_exp(k & 7);
  return x * __uint_as_float((uint32_t)(127 - 4 * e) << 23);
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

// 1 / RMS (eps 1e-6, engine/infer.js:134-143) of a residual buffer whose D / 4 quad partial sums of
// squares follow its D values; every warp forms the same sum in the same order.
__device__ __forceinline__ float inv_rms(const float* xb, int D) {
  const int lane = threadIdx.x & 31;
  float s = 0.f;
  for (int q = lane; q < D / 4; q += 32) s += xb[D + q];
  s = warp_sum(s);
  return 1.f / sqrtf(s / D + 1e-6f);
}

// Epilogue + exchange of a row stage: `val(i)` gives the value of local row i (0 .. nrows); thread i
// computes row i into stage, then thread i sends row quad i / 16 to CTA i % 16.  With ss, the quad's
// sum of squares also goes to slot (first quad + quad) after the destination's D values.
template <class F>
__device__ __forceinline__ void push_rows(int nrows, float* stage, uint32_t dst, uint32_t bar, int ss_slot0,
                                          uint32_t ss_dst, F val) {
  for (int i = threadIdx.x; i < nrows; i += kCdThreads) stage[i] = val(i);
  __syncthreads();
  for (int i = threadIdx.x; i < nrows * 4; i += kCdThreads) {
    const int q = i >> 4, d = i & 15;
    const float4 v = reinterpret_cast<const float4*>(stage)[q];
    const uint32_t rb = mapa(bar, d);
    st_async4(mapa(dst + 16 * q, d), v, rb);
    if (ss_slot0 >= 0) {
      const float s = fmaf(v.w, v.w, fmaf(v.z, v.z, fmaf(v.y, v.y, v.x * v.x)));
      st_async1(mapa(ss_dst + 4 * (ss_slot0 + q), d), s, rb);
    }
  }
}

}  // namespace cd

using namespace cd;

__global__ void __launch_bounds__(kCdThreads, 1) cdec_kernel(const __grid_constant__ CdArgs A) {
  extern __shared__ __align__(16) uint8_t smem[];
  const RunArgs& a = A.r;
  const ModelDev& md = a.m;
  const CdSmem Ls = cd_smem(md, A.smem_cap);
  const int c = (int)cta_rank();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = md.D, QKV = md.QKV, FF = md.FF, NKV = md.NKV, rep = md.NH / md.NKV;
  const int S = cd_splits(md), U = NKV * S;
  float* actp = reinterpret_cast<float*>(smem + Ls.actp);
  float* red = reinterpret_cast<float*>(smem + Ls.red);
  float* xb2 = reinterpret_cast<float*>(smem + Ls.xb2);
  float* xb1 = reinterpret_cast<float*>(smem + Ls.xb1);
  float* qkvb = reinterpret_cast<float*>(smem + Ls.qkv);
  float* hb = reinterpret_cast<float*>(smem + Ls.hb);
  float* attb = reinterpret_cast<float*>(smem + Ls.attb);
  float* cand = reinterpret_cast<float*>(smem + Ls.cand);
  float* outv = reinterpret_cast<float*>(smem + Ls.outv);
  float* wpart = reinterpret_cast<float*>(smem + Ls.wpart);
  float* qk = reinterpret_cast<float*>(smem + Ls.qk);
  float* mw = reinterpret_cast<float*>(smem + Ls.mw);
  const float** norms = reinterpret_cast<const float**>(smem + Ls.norms);
  float* misc = reinterpret_cast<float*>(smem + Ls.misc);
  int* imisc = reinterpret_cast<int*>(misc);
  const uint32_t sbar = smem_u32(smem + Ls.bars);
  const uint32_t bytes_x = (uint32_t)(D * 4 + D);  // D values + D / 4 quad sums of squares
  const uint32_t bar_bytes[B_COUNT] = {bytes_x, (uint32_t)QKV * 4, (uint32_t)(U * rep * kCdPartWords * 4), bytes_x,
                                       (uint32_t)FF * 4, (uint32_t)(kCdCtas * 16)};
  const uint64_t limit = a.wait_ns ? a.wait_ns : kWaitNs;
  uint32_t par[B_COUNT] = {0, 0, 0, 0, 0, 0};
  if (tid == 0) {
    for (int b = 0; b < B_COUNT; ++b) bar_init(sbar + 8 * b, 1);
    for (int sl = 0; sl < Ls.nslot; ++sl) bar_init(sbar + 8 * (8 + sl), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int b = 0; b < B_COUNT; ++b) bar_arm(sbar + 8 * b, bar_bytes[b]);
  }
  if (tid < 2 * kCdMaxSlots) reinterpret_cast<int*>(smem + Ls.feed)[tid] = tid < kCdMaxSlots ? 0 : -1;
  // norm gain pointers of every layer, then norm_f
  for (int i = tid; i < 2 * md.n_layers; i += kCdThreads)
    norms[i] = (i & 1) ? md.layers[i >> 1].norm2 : md.layers[i >> 1].norm1;
  if (tid == 0) norms[2 * md.n_layers] = md.norm_f;
  __syncthreads();
  cluster_sync_all();  // every barrier is armed before any CTA sends

  // bounded wait + re-arm for the next use of the same buffer
  auto wait_bar = [&](int b) -> bool {
    if (!xwait(sbar + 8 * b, par[b] & 1, a.err, limit)) return false;
    ++par[b];
    if (tid == 0) bar_arm(sbar + 8 * b, bar_bytes[b]);
    return true;
  };

  Feed F;
  F.src = A.wst + (size_t)A.woff[c] * kCdChunk;
  F.ring = smem + Ls.ring;
  F.cnt = reinterpret_cast<int*>(smem + Ls.feed);
  F.full = sbar + 8 * 8;
  F.cpt = A.wcpt[c];
  F.nslot = (uint32_t)Ls.nslot;
  F.cur = F.ring + (size_t)warp * kCdRpc * kCdRecBytes;
  F.kc = F.slot = F.phase = F.ri = 0;
  F.tok_end = F.cpt;

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
  const int off_lm = cd_stage_off(md, c, 0, CD_LM);
  const int rl = (cd_stage_off(md, c, 1, CD_QKV) - cd_stage_off(md, c, 0, CD_QKV)) & (kCdWarps - 1);  // per layer
  const int off_p = cd_stage_off(md, c, 0, CD_PROJ), off_13 = cd_stage_off(md, c, 0, CD_W13),
            off_2 = cd_stage_off(md, c, 0, CD_W2);
  // gains of this thread's elements k = tid, tid + 512 (D <= 1024): current layer and the next one
  float g1[2], g2[2], n1[2], n2[2];
  auto load_gains = [&](int l, float (&o1)[2], float (&o2)[2]) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int k = tid + kCdThreads * j;
      o1[j] = k < D ? ldv_f32(norms[2 * l] + k) : 0.f;
      o2[j] = (k < D && l < md.n_layers) ? ldv_f32(norms[2 * l + 1] + k) : 0.f;
    }
  };
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
  if (tid == 0)
    for (uint32_t k = 0; k < F.nslot; ++k) feed_issue(F, k);
  load_gains(0, n1, n2);

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
    // RoPE row of this position for the q / k element this thread rotates (threads < (rep + 1) * 64)
    float rc = 1.f, rs = 0.f;
    {
      const int d = tid & 63;
      if (tid < (rep + 1) * 64 && d < md.rope_dim) {
        rc = ldv_f32(md.rope_cos + (size_t)pos * md.rope_dim + d);
        rs = ldv_f32(md.rope_sin + (size_t)pos * md.rope_dim + d);
      }
    }
    // ---- embed (engine/infer.js:360-420): the dequantised tied lm_head row, in every CTA
    {
      const uint8_t* row = reinterpret_cast<const uint8_t*>(md.lm.w) + (size_t)tok * (D / 2);
      const float* sc = md.lm.s + (size_t)tok * (D / 32);
      for (int q = tid; q < D / 4; q += kCdThreads) {
        const uint16_t b2 = *reinterpret_cast<const uint16_t*>(row + 2 * q);
        const float s0 = sc[q >> 3];
        float v[4];
        v[0] = (float)((int)(b2 & 15) - 8) * s0;
        v[1] = (float)((int)((b2 >> 4) & 15) - 8) * s0;
        v[2] = (float)((int)((b2 >> 8) & 15) - 8) * s0;
        v[3] = (float)((int)((b2 >> 12) & 15) - 8) * s0;
        *reinterpret_cast<float4*>(xb2 + 4 * q) = make_float4(v[0], v[1], v[2], v[3]);
        xb2[D + q] = fmaf(v[3], v[3], fmaf(v[2], v[2], fmaf(v[1], v[1], v[0] * v[0])));
      }
      __syncthreads();
    }
    for (int l = 0; l < md.n_layers; ++l) {
      if (l > 0 && !(ok = wait_bar(B_X2))) goto done;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        g1[j] = n1[j];
        g2[j] = n2[j];
      }
      load_gains(l + 1 < md.n_layers ? l + 1 : l, n1, n2);
      if (l + 1 == md.n_layers) {  // the final norm's gain rides in n1
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int k = tid + kCdThreads * j;
          n1[j] = k < D ? ldv_f32(norms[2 * md.n_layers] + k) : 0.f;
        }
      }
      const float inv1 = inv_rms(xb2, D);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = tid + kCdThreads * j;
        if (k < D) actp[k] = pre_scale(xb2[k] * g1[j], k);
      }
      // attention unit of this CTA and the K/V rows its warp walks first (requested before the stage)
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
      if (!__syncthreads_and(run_units(F, gq, (l * rl) & (kCdWarps - 1), actp, red, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
      push_rows(gq.T * 16, outv, smem_u32(qkvb + 16 * gq.t0), sbar + 8 * B_QKV, -1, 0,
                [&](int i) { return inv1 * row_sum(red, gq, i); });
      if (!(ok = wait_bar(B_QKV))) goto done;
      // ---- attention of unit (kvh, sp) (engine/infer.js:442-495)
      if (has_unit) {
        // RoPE'd q heads of the group, the new k (rotated) and v (engine/infer.js:185-225)
        if (tid < (rep + 2) * 64) {
          const int vec = tid >> 6, d = tid & 63;
          const float* src = vec < rep ? qkvb + (kvh * rep + vec) * 64
                                       : vec == rep ? qkvb + D + kvh * 64 : qkvb + D + NKV * 64 + kvh * 64;
          float v = src[d];
          const int half = md.rope_dim / 2;
          if (vec <= rep && d < md.rope_dim) {
            if (d < half) v = fmaf(-src[d + half], rs, v * rc);
            else v = fmaf(src[d - half], rs, v * rc);
          }
          qk[tid] = v;
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
#pragma unroll
          for (int q = 0; q + 1 < kCdKvPre; ++q) {  // kpre[0] always belongs to the next position
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
        // per head: max over the warps, then each warp's weight exp(m_w - M); the CTA's partial is
        // (M, sum of weighted sums, 64 weighted outputs)
        if (tid < rep * 32) {
          const int h = tid >> 5, w = tid & 31;
          const float* wp = wpart + (w * rep + h) * kCdPartWords;
          const bool live = w < kCdWarps && wp[1] > 0.f;
          const float M = warp_max(live ? wp[0] : -INFINITY);
          const float wt = live ? expf(wp[0] - M) : 0.f;
          if (w < kCdWarps) mw[h * kCdWarps + w] = wt;
          const float Ls2 = warp_sum(live ? wp[1] * wt : 0.f);
          if (w == 0) {
            outv[h * kCdPartWords] = M;
            outv[h * kCdPartWords + 1] = Ls2;
            outv[h * kCdPartWords + 2] = 0.f;
            outv[h * kCdPartWords + 3] = 0.f;
          }
        }
        __syncthreads();
        if (tid < rep * 64) {
          const int h = tid >> 6, d = tid & 63;
          float O = 0.f;
          for (int w = 0; w < kCdWarps; ++w) O = fmaf(wpart[(w * rep + h) * kCdPartWords + 4 + d], mw[h * kCdWarps + w], O);
          outv[h * kCdPartWords + 4 + d] = O;
        }
        __syncthreads();
        const int n4 = rep * kCdPartWords / 4;
        const uint32_t dst = smem_u32(attb + c * rep * kCdPartWords);
        for (int i = tid; i < kCdCtas * n4; i += kCdThreads) {
          const int d = i / n4, q = i - d * n4;
          st_async4(mapa(dst + 16 * q, d), reinterpret_cast<const float4*>(outv)[q], mapa(sbar + 8 * B_ATT, d));
        }
      }
      if (!(ok = wait_bar(B_ATT))) goto done;
      // ---- merge the splits of every head: weights exp(M_s - M) / L per (head, split), then the
      // attention output straight into the proj activation
      if (tid < md.NH) {
        const int h = tid, kv = h / rep, j = h % rep;
        float M = -INFINITY;
        for (int s = 0; s < S; ++s) {
          const float* pp = attb + ((kv * S + s) * rep + j) * kCdPartWords;
          if (pp[1] > 0.f) M = fmaxf(M, pp[0]);
        }
        float Lsum = 0.f;
        for (int s = 0; s < S; ++s) {
          const float* pp = attb + ((kv * S + s) * rep + j) * kCdPartWords;
          const float wt = pp[1] > 0.f ? expf(pp[0] - M) : 0.f;
          mw[h * kCdCtas + s] = wt;
          Lsum = fmaf(pp[1], wt, Lsum);
        }
        const float inv = 1.f / Lsum;
        for (int s = 0; s < S; ++s) mw[h * kCdCtas + s] *= inv;
      }
      __syncthreads();
      for (int i = tid; i < D; i += kCdThreads) {
        const int h = i >> 6, d = i & 63, kv = h / rep, j = h % rep;
        float O = 0.f;
        for (int s = 0; s < S; ++s) O = fmaf(attb[((kv * S + s) * rep + j) * kCdPartWords + 4 + d], mw[h * kCdCtas + s], O);
        actp[i] = pre_scale(O, i);
      }
      __syncthreads();
      // ---- proj rows + residual (x1)
      if (!__syncthreads_and(run_units(F, gp, (l * rl + off_p) & (kCdWarps - 1), actp, red, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
      push_rows(gp.T * 16, outv, smem_u32(xb1 + 16 * gp.t0), sbar + 8 * B_X1, 4 * gp.t0, smem_u32(xb1 + D),
                [&](int i) { return xb2[16 * gp.t0 + i] + row_sum(red, gp, i); });
      if (!(ok = wait_bar(B_X1))) goto done;
      // ---- w1 / w3 rows, SiLU(u) * v (engine/infer.js:506-527)
      const float inv2 = inv_rms(xb1, D);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = tid + kCdThreads * j;
        if (k < D) actp[k] = pre_scale(xb1[k] * g2[j], k);
      }
      __syncthreads();
      if (!__syncthreads_and(run_units(F, gw13, (l * rl + off_13) & (kCdWarps - 1), actp, red, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
      push_rows(gw13.T * 16, outv, smem_u32(hb + 16 * gw13.t0), sbar + 8 * B_H, -1, 0, [&](int i) {
        const int tl = i >> 4, r = i & 15;
        const float u = inv2 * row_sum(red, gw13, (2 * tl) * 16 + r);
        const float v = inv2 * row_sum(red, gw13, (2 * tl + 1) * 16 + r);
        return (u / (1.f + expf(-u))) * v;
      });
      if (!(ok = wait_bar(B_H))) goto done;
      // ---- w2 rows + residual (x2)
      for (int k = tid; k < FF; k += kCdThreads) actp[k] = pre_scale(hb[k], k);
      __syncthreads();
      if (!__syncthreads_and(run_units(F, gw2, (l * rl + off_2) & (kCdWarps - 1), actp, red, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
      push_rows(gw2.T * 16, outv, smem_u32(xb2 + 16 * gw2.t0), sbar + 8 * B_X2, 4 * gw2.t0, smem_u32(xb2 + D),
                [&](int i) { return xb1[16 * gw2.t0 + i] + row_sum(red, gw2, i); });
    }
    // ---- final RMSNorm, lm_head rows of this CTA, argmax candidates (engine/infer.js:240-250)
    if (!(ok = wait_bar(B_X2))) goto done;
    {
      const float invf = inv_rms(xb2, D);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = tid + kCdThreads * j;
        if (k < D) actp[k] = pre_scale(xb2[k] * n1[j], k);
      }
      load_gains(0, n1, n2);  // the next token's first layer
      __syncthreads();
      if (!__syncthreads_and(run_units(F, glm, off_lm, actp, red, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
      if (!__syncthreads_and(feed_token_end(F, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
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
    if (c == 0 && tid == 0) {
      a.out_ids[gen] = tok;
      stream_publish(a.stream_ids, gen, tok, 1);
    }
    ++gen;
    if (tok == a.eos) stop = 0;
  }
done:
  __syncthreads();
  if (tid == 0) {
    // the bulk copies still in flight land before the CTA leaves (bounded)
    const int* last = reinterpret_cast<const int*>(smem + Ls.feed) + kCdMaxSlots;
    for (int sl = 0; sl < Ls.nslot; ++sl)
      if (last[sl] >= 0) {
        const uint32_t k = (uint32_t)last[sl];
        const uint32_t bar = sbar + 8 * (8 + sl), parity = (k / F.nslot) & 1;
        const uint64_t t0 = globaltimer();
        for (;;) {
          uint32_t done_ok;
          asm volatile(
              "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
              : "=r"(done_ok)
              : "r"(bar), "r"(parity)
              : "memory");
          if (done_ok || globaltimer() - t0 > limit) break;
        }
      }
  }
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
  if (m.NKV > kCdCtas || m.rope_dim > 64 || m.rope_dim % 2 || m.D > 2 * kCdThreads) return false;
  if ((m.NH / m.NKV + 2) * 64 > kCdThreads || m.NH > kCdThreads) return false;
  const CdSmem p = cd_smem(m, (int)smem_cap);
  return p.nslot >= 3 && (size_t)p.total <= smem_cap;
}

size_t cd_smem_bytes(const ModelDev& m, size_t smem_cap) { return (size_t)cd_smem(m, (int)smem_cap).total; }

// Records of every (CTA, warp) stream, in consumption order: per layer QKV, PROJ, W13 (w1 / w3 tiles
// interleaved), W2, then the lm_head.  A record holds, for lane = 4 gid + t, the words t of group g of
// rows gid and gid + 8 (8 bytes at 8 lane), then the scales of rows (gid, gid + 8) as a float pair at
// 256 + 8 gid.  Rows past the end hold q = 8 nibbles and zero scales.
void cd_pack(const ModelDev& m, const std::vector<HostQ4>& mats /* per layer: qkv, proj, w1, w3, w2 */,
             const HostQ4& lm, std::vector<uint8_t>* out, std::vector<uint32_t>* off, std::vector<uint32_t>* cpt,
             std::vector<uint32_t>* cnt) {
  off->assign(kCdCtas, 0);
  cpt->assign(kCdCtas, 0);
  cnt->assign(kCdCtas * kCdWarps, 0);
  auto stage_units = [&](int st, int c, int w, int off) {
    int rows, K;
    bool paired;
    cd_stage_shape(m, st, &rows, &K, &paired);
    const CdGeom g = cd_geom(rows, K, paired, c);
    const int v = (w - off) & (kCdWarps - 1);
    return (size_t)(cd_ustart(g, v + 1) - cd_ustart(g, v));
  };
  size_t chunks = 0;
  for (int c = 0; c < kCdCtas; ++c) {
    size_t mx = 0;
    for (int w = 0; w < kCdWarps; ++w) {
      size_t n = 0;
      for (int l = 0; l < m.n_layers; ++l)
        for (int st = CD_QKV; st <= CD_W2; ++st) n += stage_units(st, c, w, cd_stage_off(m, c, l, st));
      n += stage_units(CD_LM, c, w, cd_stage_off(m, c, 0, CD_LM));
      (*cnt)[c * kCdWarps + w] = (uint32_t)n;
      mx = std::max(mx, n);
    }
    (*off)[c] = (uint32_t)chunks;
    (*cpt)[c] = (uint32_t)((mx + kCdRpc - 1) / kCdRpc);
    chunks += (*cpt)[c];
  }
  out->assign(chunks * kCdChunk, 0);
  auto emit = [&](uint8_t* dst, const HostQ4& q, int r0, int g) {
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
  };
  for (int c = 0; c < kCdCtas; ++c)
    for (int w = 0; w < kCdWarps; ++w) {
      // record j of warp w goes to chunk j / kCdRpc, position w * kCdRpc + j % kCdRpc
      size_t j = 0;
      auto put = [&](const HostQ4& q, int r0, int g) {
        uint8_t* dst = out->data() + ((size_t)(*off)[c] + j / kCdRpc) * kCdChunk +
                       (size_t)(w * kCdRpc + j % kCdRpc) * kCdRecBytes;
        emit(dst, q, r0, g);
        ++j;
      };
      auto emit_stage = [&](int st, int off, const HostQ4* a, const HostQ4* b) {
        int rows, K;
        bool paired;
        cd_stage_shape(m, st, &rows, &K, &paired);
        const CdGeom g = cd_geom(rows, K, paired, c);
        const int v = (w - off) & (kCdWarps - 1);
        for (int u = cd_ustart(g, v); u < cd_ustart(g, v + 1); ++u) {
          const int tl = u / g.G, gg = u % g.G;
          const HostQ4& q = paired ? ((tl & 1) ? *b : *a) : *a;
          const int tile = g.t0 + (paired ? tl / 2 : tl);
          put(q, 16 * tile, gg);
        }
      };
      for (int l = 0; l < m.n_layers; ++l) {
        const HostQ4* L = &mats[(size_t)l * 5];
        emit_stage(CD_QKV, cd_stage_off(m, c, l, CD_QKV), &L[0], nullptr);
        emit_stage(CD_PROJ, cd_stage_off(m, c, l, CD_PROJ), &L[1], nullptr);
        emit_stage(CD_W13, cd_stage_off(m, c, l, CD_W13), &L[2], &L[3]);
        emit_stage(CD_W2, cd_stage_off(m, c, l, CD_W2), &L[4], nullptr);
      }
      emit_stage(CD_LM, cd_stage_off(m, c, 0, CD_LM), &lm, nullptr);
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
