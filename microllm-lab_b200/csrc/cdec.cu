// Cluster decode kernel: the greedy single-token decode loop of engine/infer.js:625-639 (each token is
// forwardDecode, engine/infer.js:579-601) for llama-arch files, as one thread-block cluster of 16 CTAs
// (one per SM) per kv head, resident for every token of the call.
//
// The layer is split the way tensor parallelism splits it, so that only two exchanges per layer cross
// clusters.  Cluster g owns kv head g and its rep query heads:
//
//   x -> RMSNorm -> the group's q/k/v rows (its 16 CTAs split them)   -> qkv       (DSMEM, cluster)
//   qkv -> RoPE, causal attention of the group, positions split 16 ways -> partials (DSMEM, cluster)
//   partials -> merge -> proj columns of the group's heads -> partial of all D rows
//                                                 -> x1 = x + sum of the clusters' partials   (global)
//   x1 -> RMSNorm -> w1/w3 rows of this CTA's 32-row FF slice -> SiLU(u) v (stays in the CTA)
//      -> w2 columns of the slice -> partial of all D rows -> reduce over the cluster (DSMEM)
//                                                 -> x2 = x1 + sum of the clusters' partials  (global)
// then the final RMSNorm, the lm_head rows of each CTA with a local argmax, and an exchange of the
// candidates (engine/infer.js:240-250: the lowest index wins a tie).
//
// Inside a cluster every exchange is an all-to-all through distributed shared memory: each CTA
// pushes its slice into the same buffer of all 16 CTAs with st.async, and each receiving buffer has
// an mbarrier that completes when all of the stage's bytes have landed.  Between clusters a slice is
// published as tagged 8-byte words in global memory ({tag, value}, single-copy atomic); each CTA
// polls 1/16 of the other clusters' words and forwards them by st.async to its 15 peers, so the
// words cross the L2 once per cluster.  Sums over clusters and over the CTAs of a cluster run in a
// fixed order, so the result does not depend on timing.
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
// bulk copy per chunk (cp.async.bulk of this GPU's memory, completing on the slot's mbarrier), so
// weight fetch runs layers ahead of the exchanges.  Per-layer vectors (norm gains, the RoPE row of
// the position) are fetched into registers a layer or a token ahead.
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
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
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

// Exchange barriers: x2 partials (pp2), the group's q/k/v, attention partials, x1 partials (pp1), the
// w2 reduce-scatter (rs), argmax candidates.
enum { B_X2 = 0, B_QKV = 1, B_ATT = 2, B_X1 = 3, B_RS = 4, B_CAND = 5, B_COUNT = 6 };

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
// red[(tile * maxc + slot) * 16 + row] (slot = this warp's order among the tile's warps); the warp
// that ends a tile zeroes the tile's slots after its own, so every tile holds maxc partials.  False
// when a wait for weights gave up.
// This virtual warp's units of one stage, precomputed once per launch: [u0, u1), the tile of u0 and the
// warp's slot in it (a warp that goes on into the next tile is that tile's first warp: slot 0).
struct CdRange {
  int u0, u1, tl0, slot0;
};

__device__ __forceinline__ bool run_units(Feed& F, const CdRange R, int G, int maxc, int t0, int kh, const float* actp,
                                          float* red, int warp, int lane, int* err, uint64_t limit) {
  const int gid = lane >> 2, t = lane & 3;
  if (G == 1) {
    // one group per tile: every record is its own tile, and the four lanes of a row store their
    // partials in slots t (summed by reduce_tiles), so no shuffle separates one record from the next
    const float4 a0 = reinterpret_cast<const float4*>(actp + 8 * t)[0];
    const float4 a1 = reinterpret_cast<const float4*>(actp + 8 * t)[1];
    int u = R.u0;
    while (u < R.u1) {
      if (F.ri == 0 && !feed_wait(F, err, limit)) return false;
      const int n = min(R.u1 - u, kCdRpc - (int)F.ri);
      const uint8_t* cur = F.cur;
      float* r = red + (u * 4 + t) * 16 + gid;
#pragma unroll 4
      for (int j = 0; j < n; ++j) {
        const uint2 wv = *reinterpret_cast<const uint2*>(cur + 8 * lane);
        const float2 sc = *reinterpret_cast<const float2*>(cur + 256 + 8 * gid);
        r[0] = dot8(wv.x, a0, a1) * sc.x;
        r[8] = dot8(wv.y, a0, a1) * sc.y;
        cur += kCdRecBytes;
        r += 64;
      }
      F.cur = cur;
      F.ri += n;
      u += n;
      if (F.ri == kCdRpc) feed_next_chunk(F, warp, lane);
    }
    return true;
  }
  int u = R.u0, tl = R.tl0, slot = R.slot0;
  int k = u - tl * G;  // group of the current unit within its tile
  // K halves: odd tiles start G groups into the activation
  const float* ap = actp + 32 * (k + (kh ? ((t0 + tl) & 1) * G : 0)) + 8 * t;
  float acc0 = 0.f, acc1 = 0.f;
  // the tile's partial into its slot; the warp that ends a tile zeroes the slots after its own
  auto flush = [&](bool ends_tile) {
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
    if (t == 0) {
      float* r = red + (tl * maxc + slot) * 16 + gid;
      r[0] = acc0;
      r[8] = acc1;
      if (ends_tile)
        for (int q = slot + 1; q < maxc; ++q) r[16 * (q - slot)] = r[16 * (q - slot) + 8] = 0.f;
    }
  };
  while (u < R.u1) {
    if (F.ri == 0 && !feed_wait(F, err, limit)) return false;
    // the records of this chunk that belong to the current tile: no wait or fence between them, so
    // their loads overlap the previous records' arithmetic
    const int n = min(min(R.u1 - u, G - k), kCdRpc - (int)F.ri);
    const uint8_t* cur = F.cur;
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
      const uint2 wv = *reinterpret_cast<const uint2*>(cur + 8 * lane);
      const float2 sc = *reinterpret_cast<const float2*>(cur + 256 + 8 * gid);
      const float4 a0 = reinterpret_cast<const float4*>(ap)[0];
      const float4 a1 = reinterpret_cast<const float4*>(ap)[1];
      acc0 = fmaf(dot8(wv.x, a0, a1), sc.x, acc0);
      acc1 = fmaf(dot8(wv.y, a0, a1), sc.y, acc1);
      cur += kCdRecBytes;
      ap += 32;
    }
    F.cur = cur;
    F.ri += n;
    u += n;
    k += n;
    if (F.ri == kCdRpc) feed_next_chunk(F, warp, lane);
    if (k == G) {
      flush(true);
      ++tl;
      k = 0;
      slot = 0;
      acc0 = acc1 = 0.f;
      ap = actp + 32 * (kh ? ((t0 + tl) & 1) * G : 0) + 8 * t;
    }
  }
  if (k > 0) flush(false);
  return true;
}

// Sum of each unit row's maxc partials into its slot 0, as a fixed tree over P = 2^ceil(log2 maxc)
// lanes per row (the same order on every call).  Called by the whole CTA after run_units; ends with a
// CTA barrier when there was anything to add.
__device__ __forceinline__ void reduce_tiles(float* red, const CdGeom g) {
  if (g.maxc <= 1 || g.G == 1) return;  // one-group tiles: row_val adds the four lane partials
  int lp = 1;
  while ((1 << lp) < g.maxc) ++lp;
  const int P = 1 << lp, total = g.Tu * 16 * P;
  for (int base = 0; base < total; base += kCdThreads) {
    const int t = base + (int)threadIdx.x;
    const int row = t >> lp, k = t & (P - 1);
    float* r = red + ((row >> 4) * g.maxc) * 16 + (row & 15);
    float v = (t < total && k < g.maxc) ? r[16 * k] : 0.f;
    for (int o = P >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncwarp();
    if (t < total && k == 0) r[0] = v;
  }
  __syncthreads();
}

// Row i (0 .. 16 Tu) of the CTA's unit tiles after reduce_tiles (one-group tiles: the sum of the four
// lane partials, as a fixed tree).
__device__ __forceinline__ float row_val(const float* red, const CdGeom& g, int i) {
  const float* r = red + ((i >> 4) * g.maxc) * 16 + (i & 15);
  if (g.G == 1) return (r[0] + r[16]) + (r[32] + r[48]);
  return r[0];
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

// Residual sum of this thread's elements k = tid, tid + 512 (D <= 1024): out[k] = x[k] + sum_g
// part[g D + k] (cluster order; part null: out[k] as it stands), the next stage's activation
// act[k] = pre-scaled out[k] * gain, and the warp's sum of squares into ssw[warp].  1 / RMS then
// follows from ssw after a CTA barrier (inv_rms_of).
__device__ __forceinline__ void residual_act(float* out, const float* x, const float* part, int D, int nc,
                                             const float (&gain)[2], float* act, float* ssw) {
  float s2 = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int k = (int)threadIdx.x + kCdThreads * j;
    if (k < D) {
      float v = part ? x[k] : out[k];
      if (part)
        for (int g = 0; g < nc; ++g) v += part[(size_t)g * D + k];
      out[k] = v;
      act[k] = pre_scale(v * gain[j], k);
      s2 = fmaf(v, v, s2);
    }
  }
  s2 = warp_sum(s2);
  if ((threadIdx.x & 31) == 0) ssw[threadIdx.x >> 5] = s2;
}

// 1 / RMS (eps 1e-6, engine/infer.js:134-143) from the 16 warp sums of squares; every warp forms the
// same sum in the same order.
__device__ __forceinline__ float inv_rms_of(const float* ssw, int D) {
  const int lane = threadIdx.x & 31;
  const float s = warp_sum(lane < kCdWarps ? ssw[lane] : 0.f);
  return 1.f / sqrtf(s / D + 1e-6f);
}


// Publish rows [r0, r0 + n) (n a multiple of 4) of this cluster's D-long partial vector (source slot
// `own` of nsrc; own < 0: this cluster has no partial), staged in `vals`: into the global words gx
// (several clusters), then into `part` (float index own D + r0) of every CTA of the cluster; then
// forward this CTA's 1/16 share of the other sources' vectors, as their tags arrive, to every CTA of the
// cluster.  All bytes complete on `bar` of the receiving CTA.  False when a wait for remote words gave up
// (the error flag is then raised).
__device__ __forceinline__ bool publish(const float* vals, int n, int r0, int D, int own, int nsrc, uint32_t part,
                                        uint32_t bar, uint64_t* gx, uint32_t tag, int rank, int* err,
                                        uint64_t limit) {
  if (own >= 0) {
    if (gx)
      for (int i = threadIdx.x; i < n; i += kCdThreads) ll_store(gx + (size_t)own * D + r0 + i, tag, vals[i]);
    for (int i = threadIdx.x; i < n * 4; i += kCdThreads) {  // n / 4 quads x 16 CTAs
      const int q = i >> 4, d = i & 15;
      st_async4(mapa(part + 4 * (own * D + r0 + 4 * q), d), reinterpret_cast<const float4*>(vals)[q], mapa(bar, d));
    }
  }
  if (!gx) return true;
  const int QD = D / 4, QR = (own >= 0 ? nsrc - 1 : nsrc) * QD;
  const int j1 = (rank + 1) * QR / kCdCtas;
  bool ok = true;
  for (int j = rank * QR / kCdCtas + threadIdx.x; j < j1 && ok; j += kCdThreads) {
    const int gi = j / QD, q = j - gi * QD;
    const int g = (own < 0 || gi < own) ? gi : gi + 1;
    const uint64_t* src = gx + (size_t)g * D + 4 * q;
    // the quad's four words in two 16-byte loads per round, both in flight together
    uint64_t w0, w1, w2, w3;
    const uint64_t t0 = globaltimer();
    for (int it = 0;; ++it) {
      ll_load2(src, w0, w1);
      ll_load2(src + 2, w2, w3);
      if ((uint32_t)(w0 >> 32) == tag && (uint32_t)(w1 >> 32) == tag && (uint32_t)(w2 >> 32) == tag &&
          (uint32_t)(w3 >> 32) == tag)
        break;
      if ((it & 15) == 15 && (*(volatile int*)err || globaltimer() - t0 > limit)) {
        atomicCAS(err, 0, 1);
        ok = false;
        break;
      }
    }
    if (!ok) break;
    const float v[4] = {__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1), __uint_as_float((uint32_t)w2),
                        __uint_as_float((uint32_t)w3)};
    for (int d = 0; d < kCdCtas; ++d)
      st_async4(mapa(part + 4 * (g * D + 4 * q), d), make_float4(v[0], v[1], v[2], v[3]), mapa(bar, d));
  }
  return ok;
}

}  // namespace cd

using namespace cd;

// Stage timeline (build with -DMLLM_CDEC_TIMELINE, the separate libmllm_cuda_timeline.so): thread 0 of
// every CTA stores the globaltimer at each stage boundary of one forward (mllm_timeline_config): layer
// l, stage k at word l * kCdTlLayer + k; the token's tail (final norm, lm_head, candidates) at
// kCdTlTail + k.  The stamps cost nothing in the normal build.
#ifdef MLLM_CDEC_TIMELINE
constexpr int kCdTlLayer = 24, kCdTlTail = 1000, kCdTlWords = 1024;
__device__ unsigned long long g_cd_tl[kCdMaxClusters * kCdCtas][kCdTlWords];
__device__ int g_cd_tl_forward = 3;
#define CD_TL(idx)                                                                                   \
  do {                                                                                               \
    if (tid == 0 && f == g_cd_tl_forward && (idx) < kCdTlWords) g_cd_tl[gc][(idx)] = globaltimer(); \
  } while (0)
#else
[[maybe_unused]] constexpr int kCdTlLayer = 0, kCdTlTail = 0;
#define CD_TL(idx) \
  do {             \
  } while (0)
#endif

static_assert(5 * sizeof(CdGeom) + 6 * sizeof(int) + 5 * kCdWarps * sizeof(CdRange) <= 2048, "stage table region");

__global__ void __launch_bounds__(kCdThreads, 1) cdec_kernel(const __grid_constant__ CdArgs A) {
  extern __shared__ __align__(16) uint8_t smem[];
  const RunArgs& a = A.r;
  const ModelDev& md = a.m;
  const CdSmem& Ls = A.L;
  const int nc = A.nc, nct = nc * kCdCtas, na = A.r.m.NKV;  // clusters, CTAs, attention clusters
  {
    // The launch must have the shape the weight streams were packed for: nc clusters of 16 CTAs.  A
    // launch of another shape (for example one re-issued without its cluster attribute) returns
    // before touching any stream table or peer memory, with the shape error on the flag.
    uint32_t ncta, nclu;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(ncta));
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(nclu));
    if (ncta != (uint32_t)kCdCtas || nclu != (uint32_t)nc || gridDim.x != (uint32_t)nct) {
      if (threadIdx.x == 0) atomicCAS(A.r.err, 0, kCdShapeError);
      return;
    }
  }
  const int c = (int)cta_rank();     // rank in the cluster
  const int cid = (int)cluster_id(); // the cluster's kv head (cid < na), else a helper cluster
  const bool is_attn = cid < na;
  const int gc = cid * kCdCtas + c;  // CTA of the launch
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = md.D, NKV = md.NKV, rep = md.NH / md.NKV;
  const int RO = D / kCdCtas;        // rows this CTA reduces in the w2 reduce-scatter
  float* actp = reinterpret_cast<float*>(smem + Ls.actp);
  float* red = reinterpret_cast<float*>(smem + Ls.red);
  float* xb2 = reinterpret_cast<float*>(smem + Ls.xb2);
  float* xb1 = reinterpret_cast<float*>(smem + Ls.xb1);
  float* pp1 = reinterpret_cast<float*>(smem + Ls.pp1);
  float* pp2 = reinterpret_cast<float*>(smem + Ls.pp2);
  float* rs = reinterpret_cast<float*>(smem + Ls.rs);
  float* qkvb = reinterpret_cast<float*>(smem + Ls.qkv);
  float* attb = reinterpret_cast<float*>(smem + Ls.attb);
  float* cand = reinterpret_cast<float*>(smem + Ls.cand);
  float* outv = reinterpret_cast<float*>(smem + Ls.outv);
  float* wpart = reinterpret_cast<float*>(smem + Ls.wpart);
  float* qk = reinterpret_cast<float*>(smem + Ls.qk);
  float* mw = reinterpret_cast<float*>(smem + Ls.mw);
  float* kst = reinterpret_cast<float*>(smem + Ls.kvst);  // [kCdKvStage][64]
  float* vst = kst + kCdKvStage * 64;
  const float** norms = reinterpret_cast<const float**>(smem + Ls.norms);
  float* misc = reinterpret_cast<float*>(smem + Ls.misc);
  int* imisc = reinterpret_cast<int*>(misc);
  const uint32_t sbar = smem_u32(smem + Ls.bars);
  const uint32_t kvbar = sbar + 8 * 6;
  uint32_t kvph = 0;       // phases of the K/V staging barrier completed
  bool kv_pending = false; // a staging copy is in flight
  const uint32_t bar_bytes[B_COUNT] = {(uint32_t)(nc * D * 4), (uint32_t)(2 * (rep + 2) * 64 * 4),
                                       (uint32_t)(kCdCtas * rep * kCdPartWords * 4), (uint32_t)(na * D * 4),
                                       (uint32_t)(D * 4), (uint32_t)(nct * 16)};
  const uint64_t limit = a.wait_ns ? a.wait_ns : kWaitNs;
  uint32_t par[B_COUNT] = {0, 0, 0, 0, 0, 0};
  if (tid == 0) {
    for (int b = 0; b < B_COUNT; ++b) bar_init(sbar + 8 * b, 1);
    bar_init(kvbar, 1);
    for (int sl = 0; sl < Ls.nslot; ++sl) bar_init(sbar + 8 * (8 + sl), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int b = 0; b < B_COUNT; ++b) bar_arm(sbar + 8 * b, bar_bytes[b]);
  }
  if (tid < 2 * kCdMaxSlots) reinterpret_cast<int*>(smem + Ls.feed)[tid] = tid < kCdMaxSlots ? 0 : -1;
  // norm gain pointers of every layer, then norm_f
  for (int i = tid; i < 2 * md.n_layers; i += kCdThreads)
    norms[i] = (i & 1) ? md.layers[i >> 1].norm2 : md.layers[i >> 1].norm1;
  if (tid == 0) norms[2 * md.n_layers] = md.norm_f;
  // per stage: this CTA's geometry and the rotation offset of layer 0; then the offset's step per layer
  CdGeom* geo = reinterpret_cast<CdGeom*>(smem + Ls.geo);  // [5]
  int* offs = reinterpret_cast<int*>(geo + 5);              // [6]
  CdRange* wr = reinterpret_cast<CdRange*>(offs + 6);       // [5][16]: per stage and virtual warp
  if (tid < 5 * kCdWarps) {
    const int st = tid / kCdWarps, v = tid % kCdWarps;
    const CdGeom g = cd_stage_geom(md, st, cid, c, nc);
    CdRange r;
    r.u0 = cd_ustart(g, v);
    r.u1 = cd_ustart(g, v + 1);
    r.tl0 = g.G > 0 ? r.u0 / g.G : 0;
    r.slot0 = r.u0 < r.u1 ? v - cd_vwarp(g, r.tl0 * g.G) : 0;
    wr[tid] = r;
  }
  if (tid < 5) {
    geo[tid] = cd_stage_geom(md, tid, cid, c, nc);
    offs[tid] = cd_stage_off(md, cid, c, nc, 0, tid);
    if (tid == 0) offs[5] = (cd_stage_off(md, cid, c, nc, 1, CD_QKV) - cd_stage_off(md, cid, c, nc, 0, CD_QKV)) &
                            (kCdWarps - 1);
  }
  __syncthreads();
  cluster_sync_all();  // every barrier is armed before any CTA sends
  const CdGeom& gq = geo[CD_QKV];
  const CdGeom& gp = geo[CD_PROJ];
  const CdGeom& gw13 = geo[CD_W13];
  const CdGeom& gw2 = geo[CD_W2];
  const CdGeom& glm = geo[CD_LM];
  const int rl = offs[5];
  const int off_p = offs[CD_PROJ], off_13 = offs[CD_W13], off_2 = offs[CD_W2], off_lm = offs[CD_LM];

  // bounded wait + re-arm for the next use of the same buffer
  auto wait_bar = [&](int b) -> bool {
    if (!xwait(sbar + 8 * b, par[b] & 1, a.err, limit)) return false;
    ++par[b];
    if (tid == 0) bar_arm(sbar + 8 * b, bar_bytes[b]);
    return true;
  };
  // global exchange words of a buffer for its current use (null with one cluster), and the use's tag
  auto gxb = [&](int gb, int b) -> uint64_t* {
    if (nc == 1) return nullptr;
    const size_t words = (cd_gx_words(md, nc, gb + 1) - cd_gx_words(md, nc, gb)) / 2;
    return A.gx + cd_gx_words(md, nc, gb) + (par[b] & 1) * words;
  };
  auto tagb = [&](int b) { return A.tag0 + 1u + par[b]; };

  Feed F;
  F.src = A.wst + (size_t)A.woff[gc] * kCdChunk;
  F.ring = smem + Ls.ring;
  F.cnt = reinterpret_cast<int*>(smem + Ls.feed);
  F.full = sbar + 8 * 8;
  F.cpt = A.wcpt[gc];
  F.nslot = (uint32_t)Ls.nslot;
  F.cur = F.ring + (size_t)warp * kCdRpc * kCdRecBytes;
  F.kc = F.slot = F.phase = F.ri = 0;
  F.tok_end = F.cpt;
  // Copy the first nst cache rows (K and V) of this CTA's positions [p0, ..) of `layer` into shared
  // memory (one thread issues; every thread records the pending phase).  The issuing thread's proxy
  // fence orders the cache rows other CTAs of the cluster stored (seen through the cluster's
  // release/acquire exchanges) and this CTA's earlier reads of the buffers before the copies.
  auto stage_kv = [&](int layer, int p0, int nst, bool issuer) {
    if (nst <= 0) return;
    if (issuer) {
      const size_t base = ((size_t)layer * md.NKV + cid) * md.kv_len + p0;
      asm volatile("fence.proxy.async;" ::: "memory");
      bar_arm(kvbar, 2u * nst * 256u);
      bulk_g2s(kst, a.kc + base * 64, nst * 256u, reinterpret_cast<uint64_t*>(smem + Ls.bars) + 6);
      bulk_g2s(vst, a.vc + base * 64, nst * 256u, reinterpret_cast<uint64_t*>(smem + Ls.bars) + 6);
    }
    kv_pending = true;
  };
  // this warp's share of stage st when the stage's rotation offset is off
  auto units = [&](int st, int off) {
    return run_units(F, wr[st * kCdWarps + ((warp - off) & (kCdWarps - 1))], geo[st].G, geo[st].maxc, geo[st].t0,
                     geo[st].kh, actp, red, warp, lane, a.err, limit);
  };

  const bool gen_mode = a.mode == MODE_GENERATE;
  int gen = 0, tok = 0, stop = 1, f = 0;
  bool ok = true;
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
    float rc = 1.f, rs_ = 0.f;
    {
      const int d = tid & 63;
      if (tid < (rep + 1) * 64 && d < md.rope_dim) {
        rc = ldv_f32(md.rope_cos + (size_t)pos * md.rope_dim + d);
        rs_ = ldv_f32(md.rope_sin + (size_t)pos * md.rope_dim + d);
      }
    }
    // ---- embed (engine/infer.js:360-420): the dequantised tied lm_head row, this thread's elements
    {
      const uint8_t* row = reinterpret_cast<const uint8_t*>(md.lm.w) + (size_t)tok * (D / 2);
      const float* sc = md.lm.s + (size_t)tok * (D / 32);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k = tid + kCdThreads * j;
        if (k < D) {
          const int b = row[k >> 1];  // element 2i in the low nibble of byte i, 2i + 1 in the high one
          xb2[k] = (float)(((k & 1) ? (b >> 4) : (b & 15)) - 8) * sc[k >> 5];
        }
      }
    }
    for (int l = 0; l < md.n_layers; ++l) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        g1[j] = n1[j];
        g2[j] = n2[j];
      }
      CD_TL(l * kCdTlLayer + 0);
      if (l > 0) {  // x2 of the previous layer
        if (!(ok = wait_bar(B_X2))) goto done;
        residual_act(xb2, xb1, pp2, D, nc, g1, actp, misc);
        CD_TL(l * kCdTlLayer + 1);
      } else {
        residual_act(xb2, nullptr, nullptr, D, nc, g1, actp, misc);
        CD_TL(l * kCdTlLayer + 1);
      }
      load_gains(l + 1 < md.n_layers ? l + 1 : l, n1, n2);
      if (l + 1 == md.n_layers) {  // the final norm's gain rides in n1
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int k = tid + kCdThreads * j;
          n1[j] = k < D ? ldv_f32(norms[2 * md.n_layers] + k) : 0.f;
        }
      }
      // this CTA's split of the positions [p_lo, p_hi); its first kCdKvStage cache rows are copied into
      // shared memory now, so that they have landed when attention starts
      const int span = (pos + kCdCtas) / kCdCtas;
      const int p_lo = c * span, p_hi = min(pos + 1, p_lo + span);
      const int npos = max(0, p_hi - p_lo);
      const int nst = max(0, min(min(p_hi, pos) - p_lo, kCdKvStage));
      const size_t kv_base = ((size_t)l * NKV + cid) * md.kv_len;
      if (l == 0 && is_attn) stage_kv(0, p_lo, nst, tid == 0);
      __syncthreads();
      const float inv1 = inv_rms_of(misc, D);
      CD_TL(l * kCdTlLayer + 2);
      if (is_attn) {  // ---- attention clusters: q/k/v, attention and the proj columns of the group
      // ---- the group's q/k/v rows (engine/infer.js:431-440)
      if (!__syncthreads_and(units(CD_QKV, l * rl))) {
        ok = false;
        goto done;
      }
      reduce_tiles(red, gq);
      for (int i = tid; i < gq.T * 16; i += kCdThreads) outv[i] = inv1 * row_val(red, gq, i);
      CD_TL(l * kCdTlLayer + 3);
      __syncthreads();
      for (int i = tid; i < gq.T * 16 * 4; i += kCdThreads) {  // quads x 16 CTAs
        const int q = i >> 4, d = i & 15;
        const int j = gq.t0 + (q >> 2);  // K half j % 2 of group-local tile j / 2
        st_async4(mapa(smem_u32(qkvb + (j & 1) * (rep + 2) * 64 + 16 * (j >> 1) + 4 * (q & 3)), d),
                  reinterpret_cast<const float4*>(outv)[q], mapa(sbar + 8 * B_QKV, d));
      }
      CD_TL(l * kCdTlLayer + 4);
      if (!(ok = wait_bar(B_QKV))) goto done;
      CD_TL(l * kCdTlLayer + 5);
      // ---- attention of the group over this CTA's positions (engine/infer.js:442-495)
      {
        // RoPE'd q heads of the group, the new k (rotated) and v (engine/infer.js:185-225)
        if (tid < (rep + 2) * 64) {
          const int vec = tid >> 6, d = tid & 63;
          const float* src = qkvb + vec * 64;
          const float* src2 = src + (rep + 2) * 64;  // the second K half
          float v = src[d] + src2[d];
          const int half = md.rope_dim / 2;
          if (vec <= rep && d < md.rope_dim) {
            if (d < half) v = fmaf(-(src[d + half] + src2[d + half]), rs_, v * rc);
            else v = fmaf(src[d - half] + src2[d - half], rs_, v * rc);
          }
          qk[tid] = v;
        }
        __syncthreads();
        CD_TL(l * kCdTlLayer + 6);
        // every position of the CTA in the staged rows: the new row is copied in beside them
        const bool fast = npos <= kCdKvStage;
        if (pos >= p_lo && pos < p_hi && tid < 128) {  // the cache row (engine/infer.js:457-464)
          const int d = tid & 63;
          if (tid < 64) {
            const float v = qk[rep * 64 + d];
            a.kc[(kv_base + pos) * 64 + d] = v;
            if (fast) kst[(pos - p_lo) * 64 + d] = v;
          } else {
            const float v = qk[(rep + 1) * 64 + d];
            a.vc[(kv_base + pos) * 64 + d] = v;
            if (fast) vst[(pos - p_lo) * 64 + d] = v;
          }
        }
        if (nst > 0) {
          if (!mbar_wait_bounded(reinterpret_cast<uint64_t*>(smem + Ls.bars) + 6, kvph & 1, limit)) atomicCAS(a.err, 0, 1);
          ++kvph;
          kv_pending = false;
        }
        __syncthreads();
        CD_TL(l * kCdTlLayer + 7);
        if (fast) {
          // warp h scores head h: lane j takes position p_lo + j (q . k over the 64 dims, read in a rotated
          // order so that the lanes' rows fall in different banks); then the softmax weights scale the v
          // rows, each lane owning two of the 64 outputs
          if (warp < rep) {
            const float* qh = qk + warp * 64;
            float s = -INFINITY;
            if (lane < npos) {
              float acc[4] = {0.f, 0.f, 0.f, 0.f};
              const float* kr = kst + lane * 64;
#pragma unroll 4
              for (int d4 = 0; d4 < 16; ++d4) {
                const int d = ((d4 + lane) & 15) * 4;
                const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
                const float4 q4 = *reinterpret_cast<const float4*>(qh + d);
                acc[d4 & 3] = fmaf(q4.w, k4.w, fmaf(q4.z, k4.z, fmaf(q4.y, k4.y, fmaf(q4.x, k4.x, acc[d4 & 3]))));
              }
              s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * 0.125f;  // 1/sqrt(64)
            }
            const float mx = warp_max(s);
            const float e = lane < npos ? expf(s - mx) : 0.f;
            const float lsum = warp_sum(e);
            float o0 = 0.f, o1 = 0.f;
#pragma unroll 4
            for (int jj = 0; jj < npos; ++jj) {
              const float w = __shfl_sync(0xffffffffu, e, jj);
              const float2 v2 = *reinterpret_cast<const float2*>(vst + jj * 64 + 2 * lane);
              o0 = fmaf(w, v2.x, o0);
              o1 = fmaf(w, v2.y, o1);
            }
            float* op = outv + warp * kCdPartWords;
            if (lane == 0) {
              op[0] = mx;
              op[1] = lsum;
              op[2] = op[3] = 0.f;
            }
            op[4 + 2 * lane] = o0;
            op[5 + 2 * lane] = o1;
          }
        } else {
        // Warp w takes head h = w % rep and every nwh-th chunk of 32 positions from chunk w / rep; lane j
        // of a chunk scores position p_lo + chunk start + j (q . k over the 64 dims, read in a rotated
        // order so that the lanes' rows fall in different banks), then the chunk's softmax weights scale
        // the v rows, each lane owning two of the 64 outputs (online softmax across chunks).
        const int nwh = kCdWarps / rep, h = warp % rep, sub = warp / rep;
        float m = -INFINITY, lsum = 0.f, o0 = 0.f, o1 = 0.f;
        if (sub < nwh) {
          const float* qh = qk + h * 64;
          for (int c0 = 32 * sub; c0 < npos; c0 += 32 * nwh) {
            const int j = c0 + lane, p = p_lo + j;
            float s = -INFINITY;
            if (j < npos) {
              float acc[4] = {0.f, 0.f, 0.f, 0.f};
              if (p == pos || j < nst) {
                const float* kr = p == pos ? qk + rep * 64 : kst + j * 64;
#pragma unroll 4
                for (int d4 = 0; d4 < 16; ++d4) {
                  const int d = ((d4 + lane) & 15) * 4;
                  const float4 k4 = *reinterpret_cast<const float4*>(kr + d);
                  const float4 q4 = *reinterpret_cast<const float4*>(qh + d);
                  acc[d4 & 3] = fmaf(q4.w, k4.w, fmaf(q4.z, k4.z, fmaf(q4.y, k4.y, fmaf(q4.x, k4.x, acc[d4 & 3]))));
                }
              } else {
                const float* kr = a.kc + (kv_base + p) * 64;
#pragma unroll 4
                for (int d4 = 0; d4 < 16; ++d4) {
                  const float4 k4 = ldcg_f4(kr + 4 * d4);
                  const float4 q4 = *reinterpret_cast<const float4*>(qh + 4 * d4);
                  acc[d4 & 3] = fmaf(q4.w, k4.w, fmaf(q4.z, k4.z, fmaf(q4.y, k4.y, fmaf(q4.x, k4.x, acc[d4 & 3]))));
                }
              }
              s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) * 0.125f;  // 1/sqrt(64)
            }
            const float nm = fmaxf(m, warp_max(s));
            const float corr = m == -INFINITY ? 0.f : expf(m - nm);
            const float e = j < npos ? expf(s - nm) : 0.f;
            lsum = fmaf(lsum, corr, warp_sum(e));
            o0 *= corr;
            o1 *= corr;
            const int cnt = min(32, npos - c0);
            for (int jj = 0; jj < cnt; ++jj) {
              const float w = __shfl_sync(0xffffffffu, e, jj);
              const int q = c0 + jj, pq = p_lo + q;
              float2 v2;
              if (pq == pos) v2 = *reinterpret_cast<const float2*>(qk + (rep + 1) * 64 + 2 * lane);
              else if (q < nst) v2 = *reinterpret_cast<const float2*>(vst + q * 64 + 2 * lane);
              else v2 = ldcg_f2(a.vc + (kv_base + pq) * 64 + 2 * lane);
              o0 = fmaf(w, v2.x, o0);
              o1 = fmaf(w, v2.y, o1);
            }
            m = nm;
          }
        }
        // the CTA's partial per head (max, sum, 64 weighted outputs), combined over the head's warps
        {
          const int nsub = min(nwh, (npos + 31) / 32);
          if (sub < nwh) {
            float* wp = wpart + (sub * rep + h) * kCdPartWords;
            if (lane == 0) {
              wp[0] = m;
              wp[1] = lsum;
            }
            wp[4 + 2 * lane] = o0;
            wp[5 + 2 * lane] = o1;
          }
          __syncthreads();
          if (tid < rep * 32) {
            const int hh = tid >> 5, w = tid & 31;
            const float* wp = wpart + (w * rep + hh) * kCdPartWords;
            const bool live = w < nsub && wp[1] > 0.f;
            const float M = warp_max(live ? wp[0] : -INFINITY);
            const float wt = live ? expf(wp[0] - M) : 0.f;
            if (w < kCdWarps) mw[hh * kCdWarps + w] = wt;
            const float Ls2 = warp_sum(live ? wp[1] * wt : 0.f);
            if (w == 0) {
              outv[hh * kCdPartWords] = M;
              outv[hh * kCdPartWords + 1] = Ls2;
              outv[hh * kCdPartWords + 2] = 0.f;
              outv[hh * kCdPartWords + 3] = 0.f;
            }
          }
          __syncthreads();
          if (tid < rep * 64) {
            const int hh = tid >> 6, d = tid & 63;
            float O = 0.f;
            for (int w = 0; w < nsub; ++w) O = fmaf(wpart[(w * rep + hh) * kCdPartWords + 4 + d], mw[hh * kCdWarps + w], O);
            outv[hh * kCdPartWords + 4 + d] = O;
          }
        }
        }
        __syncthreads();
        CD_TL(l * kCdTlLayer + 8);
        // the staged rows are read: the next layer's rows go in now, from a thread of the last warp
        if (l + 1 < md.n_layers) stage_kv(l + 1, p_lo, nst, tid == kCdThreads - 1);
        const int n4 = rep * kCdPartWords / 4;
        const uint32_t dst = smem_u32(attb + c * rep * kCdPartWords);
        for (int i = tid; i < kCdCtas * n4; i += kCdThreads) {
          const int d = i / n4, q = i - d * n4;
          st_async4(mapa(dst + 16 * q, d), reinterpret_cast<const float4*>(outv)[q], mapa(sbar + 8 * B_ATT, d));
        }
      }
      CD_TL(l * kCdTlLayer + 9);
      if (!(ok = wait_bar(B_ATT))) goto done;
      CD_TL(l * kCdTlLayer + 10);
      // ---- merge the 16 splits of each head: weights exp(M_s - M) / L, then the group's attention
      // output straight into the proj activation
      // splits that hold positions: CTA s covers [s span, (s + 1) span)
      const int nsp = min(kCdCtas, pos / span + 1);
      if (warp < rep) {  // warp h: the weights of head h's splits (lane s)
        const int h = warp, s = lane;
        const float* pp = attb + (s * rep + h) * kCdPartWords;
        const bool live = s < nsp && pp[1] > 0.f;
        const float M = warp_max(live ? pp[0] : -INFINITY);
        const float wt = live ? expf(pp[0] - M) : 0.f;
        const float inv = 1.f / warp_sum(live ? pp[1] * wt : 0.f);
        if (s < kCdCtas) mw[h * kCdCtas + s] = wt * inv;
      }
      __syncthreads();
      if (tid < 2 * rep * 64) {  // output i = tid / 2: even splits on one lane, odd on the next
        const int i = tid >> 1, h = i >> 6, d = i & 63;
        float O = 0.f;
        for (int s = tid & 1; s < nsp; s += 2) O = fmaf(attb[(s * rep + h) * kCdPartWords + 4 + d], mw[h * kCdCtas + s], O);
        O += __shfl_xor_sync(0xffffffffu, O, 1);
        if ((tid & 1) == 0) actp[i] = pre_scale(O, i);
      }
      __syncthreads();
      // ---- proj columns of the group -> partial rows -> x1 (engine/infer.js:497-504)
      CD_TL(l * kCdTlLayer + 11);
      if (!__syncthreads_and(units(CD_PROJ, l * rl + off_p))) {
        ok = false;
        goto done;
      }
      reduce_tiles(red, gp);
      for (int i = tid; i < gp.T * 16; i += kCdThreads) outv[i] = row_val(red, gp, i);
      CD_TL(l * kCdTlLayer + 12);
      __syncthreads();
      }
      // a remote wait that gives up raises the error flag; the wait that follows then fails everywhere
      // (helper clusters only forward the attention clusters' partials)
      (void)publish(outv, gp.T * 16, 16 * gp.t0, D, is_attn ? cid : -1, na, smem_u32(pp1), sbar + 8 * B_X1,
                    gxb(CD_GX_PP1, B_X1), tagb(B_X1), c, a.err, limit);
      CD_TL(l * kCdTlLayer + 13);
      if (!(ok = wait_bar(B_X1))) goto done;
      CD_TL(l * kCdTlLayer + 14);
      residual_act(xb1, xb2, pp1, D, na, g2, actp, misc);
      __syncthreads();
      // ---- w1 / w3 rows of this CTA's FF slice, SiLU(u) * v (engine/infer.js:506-527)
      const float inv2 = inv_rms_of(misc, D);
      CD_TL(l * kCdTlLayer + 15);
      if (!__syncthreads_and(units(CD_W13, l * rl + off_13))) {
        ok = false;
        goto done;
      }
      CD_TL(l * kCdTlLayer + 16);
      reduce_tiles(red, gw13);
      // the w2 activation: this CTA's h values at their place in its 32-column groups (k0 = s0 / 2), zero
      // in the half group that belongs to the neighbouring CTA
      for (int i = tid; i < 32 * gw2.G; i += kCdThreads) {
        const int k = i - 16 * (gw13.t0 & 1);  // h row of this CTA's slices
        float hv = 0.f;
        if (k >= 0 && k < 16 * gw13.T) {
          const int tl = k >> 4, r = k & 15;
          const float u = inv2 * row_val(red, gw13, (2 * tl) * 16 + r);
          const float v = inv2 * row_val(red, gw13, (2 * tl + 1) * 16 + r);
          hv = (u / (1.f + expf(-u))) * v;
        }
        actp[i] = pre_scale(hv, i);
      }
      __syncthreads();
      // ---- w2 columns of the slice -> partial of all D rows -> reduce over the cluster -> x2
      CD_TL(l * kCdTlLayer + 17);
      if (!__syncthreads_and(units(CD_W2, l * rl + off_2))) {
        ok = false;
        goto done;
      }
      reduce_tiles(red, gw2);
      for (int i = tid; i < D; i += kCdThreads) outv[i] = gw2.G > 0 ? row_val(red, gw2, i) : 0.f;
      CD_TL(l * kCdTlLayer + 18);
      __syncthreads();
      for (int i = tid; i < D / 4; i += kCdThreads) {  // quad i goes to the CTA that reduces its rows
        const int d = (4 * i) / RO, k = 4 * i - d * RO;
        st_async4(mapa(smem_u32(rs + c * RO + k), d), reinterpret_cast<const float4*>(outv)[i],
                  mapa(sbar + 8 * B_RS, d));
      }
      CD_TL(l * kCdTlLayer + 19);
      if (!(ok = wait_bar(B_RS))) goto done;
      CD_TL(l * kCdTlLayer + 20);
      if (tid < 8 * RO) {  // row tid / 8: lane k adds the partials of CTAs k and k + 8, then a tree over the 8 lanes
        const int i = tid >> 3, k = tid & 7;
        float s = rs[k * RO + i] + rs[(k + 8) * RO + i];
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (k == 0) outv[i] = s;
      }
      __syncthreads();
      (void)publish(outv, RO, c * RO, D, cid, nc, smem_u32(pp2), sbar + 8 * B_X2, gxb(CD_GX_PP2, B_X2), tagb(B_X2), c,
                    a.err, limit);
      CD_TL(l * kCdTlLayer + 21);
    }
    // ---- final RMSNorm, lm_head rows of this CTA, argmax candidates (engine/infer.js:240-250)
    CD_TL(kCdTlTail + 0);
    if (!(ok = wait_bar(B_X2))) goto done;
    residual_act(xb2, xb1, pp2, D, nc, n1, actp, misc);
    load_gains(0, n1, n2);  // the next token's first layer
    __syncthreads();
    {
      const float invf = inv_rms_of(misc, D);
      CD_TL(kCdTlTail + 1);
      if (!__syncthreads_and(units(CD_LM, off_lm))) {
        ok = false;
        goto done;
      }
      CD_TL(kCdTlTail + 2);
      if (!__syncthreads_and(feed_token_end(F, warp, lane, a.err, limit))) {
        ok = false;
        goto done;
      }
      reduce_tiles(red, glm);
      float best = -INFINITY;
      int bidx = 0x7fffffff;
      const int r0 = 16 * glm.t0;
      for (int i = tid; i < glm.T * 16; i += kCdThreads) {
        const int r = r0 + i;
        if (r >= md.vocab) break;
        const float v = invf * row_val(red, glm, i);
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
      // this CTA's candidate: to every CTA of the cluster directly, and (several clusters) to gx,
      // from where each CTA forwards its 1/16 share of the other clusters' candidates
      uint64_t* gcand = gxb(CD_GX_CAND, B_CAND);
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
        if (gcand && tid == 0) {
          ll_store(gcand + 2 * gc, tagb(B_CAND), bv);
          ll_store_u32(gcand + 2 * gc + 1, tagb(B_CAND), (uint32_t)bi);
        }
        st_async4(mapa(smem_u32(cand + 4 * gc), tid), make_float4(bv, __int_as_float(bi), 0.f, 0.f),
                  mapa(sbar + 8 * B_CAND, tid));
      }
      if (gcand) {
        // other clusters' CTAs: [0, 16 cid) and [16 cid + 16, nct); this CTA takes 1/16 of them
        const int nr = nct - kCdCtas;
        bool cok = true;
        for (int j = c * nr / kCdCtas + tid; j < (c + 1) * nr / kCdCtas && cok; j += kCdThreads) {
          const int g = j < cid * kCdCtas ? j : j + kCdCtas;
          uint64_t w0 = 0, w1 = 0;
          const uint64_t t0 = globaltimer();
          for (int n = 0;; ++n) {
            ll_load2(gcand + 2 * g, w0, w1);
            if ((uint32_t)(w0 >> 32) == tagb(B_CAND) && (uint32_t)(w1 >> 32) == tagb(B_CAND)) break;
            if ((n & 15) == 15 && (*(volatile int*)a.err || globaltimer() - t0 > limit)) {
              atomicCAS(a.err, 0, 1);
              cok = false;
              break;
            }
          }
          if (!cok) break;
          for (int d = 0; d < kCdCtas; ++d)
            st_async4(mapa(smem_u32(cand + 4 * g), d),
                      make_float4(__uint_as_float((uint32_t)w0), __uint_as_float((uint32_t)w1), 0.f, 0.f),
                      mapa(sbar + 8 * B_CAND, d));
        }
      }
      CD_TL(kCdTlTail + 3);
      if (!(ok = wait_bar(B_CAND))) goto done;
      CD_TL(kCdTlTail + 4);
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int cc = 0; cc < nct; ++cc) {
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
      if (gc == 0 && tid == 0 && a.argmax_out) a.argmax_out[0] = tok;
      continue;
    }
    if (gc == 0 && tid == 0) {
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
    if (kv_pending) (void)mbar_wait_bounded(reinterpret_cast<uint64_t*>(smem + Ls.bars) + 6, kvph & 1, limit);
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
  if (gc == 0 && tid == 0 && a.mode != MODE_SELFTEST_WAIT && ok) {
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
// head, at most kCdMaxClusters kv heads (one cluster each), FF a whole number of 32-row slices, an
// lm_head tile for every CTA, and the shared-memory plan within `smem_cap` with at least two ring
// slots.
bool cd_supported(const ModelDev& m, size_t smem_cap, int nc) {
  if (m.arch != 0 || m.D != m.NH * 64 || m.NH % m.NKV || m.NH / m.NKV > 4) return false;
  if (m.NKV < 1 || m.NKV > kCdMaxClusters || m.FF % 32 || m.D > 2 * kCdThreads) return false;
  if (m.rope_dim > 64 || m.rope_dim % 2) return false;
  if (nc < m.NKV || nc > kCdMaxClusters || (m.vocab + 15) / 16 < nc * kCdCtas) return false;
  const CdSmem p = cd_smem(m, (int)smem_cap, nc);
  return p.nslot >= 2 && (size_t)p.total <= smem_cap;
}

size_t cd_smem_bytes(const ModelDev& m, size_t smem_cap, int nc) {
  return (size_t)cd_smem(m, (int)smem_cap, nc).total;
}

// Records of every (CTA, warp) stream, in consumption order: per layer QKV, PROJ, W13 (w1 / w3 tiles
// interleaved), W2, then the lm_head.  A record holds, for lane = 4 gid + t, the words t of group g of
// rows gid and gid + 8 (8 bytes at 8 lane), then the scales of rows (gid, gid + 8) as a float pair at
// 256 + 8 gid.  Rows past the end hold q = 8 nibbles and zero scales.
void cd_pack(const ModelDev& m, int nc, const std::vector<HostQ4>& mats /* per layer: qkv, proj, w1, w3, w2 */,
             const HostQ4& lm, std::vector<uint8_t>* out, std::vector<uint32_t>* off, std::vector<uint32_t>* cpt,
             std::vector<uint32_t>* cnt) {
  const int nct = nc * kCdCtas;
  off->assign(nct, 0);
  cpt->assign(nct, 0);
  cnt->assign((size_t)nct * kCdWarps, 0);
  auto stage_units = [&](int st, int cid, int c, int w, int o) {
    const CdGeom g = cd_stage_geom(m, st, cid, c, nc);
    const int v = (w - o) & (kCdWarps - 1);
    return (size_t)(cd_ustart(g, v + 1) - cd_ustart(g, v));
  };
  size_t chunks = 0;
  for (int gc = 0; gc < nct; ++gc) {
    const int cid = gc / kCdCtas, c = gc % kCdCtas;
    size_t mx = 0;
    for (int w = 0; w < kCdWarps; ++w) {
      size_t n = 0;
      for (int l = 0; l < m.n_layers; ++l)
        for (int st = CD_QKV; st <= CD_W2; ++st) n += stage_units(st, cid, c, w, cd_stage_off(m, cid, c, nc, l, st));
      n += stage_units(CD_LM, cid, c, w, cd_stage_off(m, cid, c, nc, 0, CD_LM));
      (*cnt)[gc * kCdWarps + w] = (uint32_t)n;
      mx = std::max(mx, n);
    }
    (*off)[gc] = (uint32_t)chunks;
    (*cpt)[gc] = (uint32_t)((mx + kCdRpc - 1) / kCdRpc);
    chunks += (*cpt)[gc];
  }
  out->assign(chunks * kCdChunk, 0);
  // wmask: bit t keeps word t (columns 8t .. 8t + 7 of the group); masked words hold weight 0
  auto emit = [&](uint8_t* dst, const HostQ4& q, int r0, int g, unsigned wmask) {
    const int hb = q.K / 2, ng = q.K / 32;
    for (int lane = 0; lane < 32; ++lane) {
      const int gid = lane >> 2, t = lane & 3;
      for (int h = 0; h < 2; ++h) {
        const int r = r0 + gid + 8 * h;
        uint32_t word = 0x88888888u;
        if (r < q.rows && ((wmask >> t) & 1)) memcpy(&word, q.w + (size_t)r * hb + 16 * g + 4 * t, 4);
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
  for (int gc = 0; gc < nct; ++gc) {
    const int cid = gc / kCdCtas, c = gc % kCdCtas;
    for (int w = 0; w < kCdWarps; ++w) {
      // record j of warp w goes to chunk j / kCdRpc, position w * kCdRpc + j % kCdRpc
      size_t j = 0;
      auto put = [&](const HostQ4& q, int r0, int g, unsigned wmask = 15u) {
        uint8_t* dst = out->data() + ((size_t)(*off)[gc] + j / kCdRpc) * kCdChunk +
                       (size_t)(w * kCdRpc + j % kCdRpc) * kCdRecBytes;
        emit(dst, q, r0, g, wmask);
        ++j;
      };
      auto emit_stage = [&](int st, int l, const HostQ4* a, const HostQ4* b) {
        const CdGeom g = cd_stage_geom(m, st, cid, c, nc);
        const int v = (w - cd_stage_off(m, cid, c, nc, l, st)) & (kCdWarps - 1);
        for (int u = cd_ustart(g, v); u < cd_ustart(g, v + 1); ++u) {
          const int tl = u / g.G, gg = g.k0 + u % g.G;
          if (st == CD_QKV) {
            put(*a, cd_qkv_row(m, cid, (g.t0 + tl) >> 1), gg + ((g.t0 + tl) & 1) * g.G);
          } else if (st == CD_W13) {
            put((tl & 1) ? *b : *a, 16 * (g.t0 + tl / 2), gg);
          } else if (st == CD_W2) {  // only this CTA's h columns [16 s0, 16 s1) of group gg
            int s0, s1;
            cd_ff_slices(m, gc, nct, &s0, &s1);
            unsigned wmask = 0;
            for (int t = 0; t < 4; ++t) {
              const int k = 32 * gg + 8 * t;
              if (k >= 16 * s0 && k < 16 * s1) wmask |= 1u << t;
            }
            put(*a, 16 * (g.t0 + tl), gg, wmask);
          } else {
            put(*a, 16 * (g.t0 + tl), gg);
          }
        }
      };
      for (int l = 0; l < m.n_layers; ++l) {
        const HostQ4* L = &mats[(size_t)l * 5];
        emit_stage(CD_QKV, l, &L[0], nullptr);
        emit_stage(CD_PROJ, l, &L[1], nullptr);
        emit_stage(CD_W13, l, &L[2], &L[3]);
        emit_stage(CD_W2, l, &L[4], nullptr);
      }
      emit_stage(CD_LM, 0, &lm, nullptr);
    }
  }
}

#ifdef MLLM_CDEC_TIMELINE
// Timeline build only: which forward of a launch is stamped, and the stamps of the first `ctas` CTAs.
extern "C" int mllm_timeline_config(int forward) {
  return (int)cudaMemcpyToSymbol(g_cd_tl_forward, &forward, sizeof(int));
}
extern "C" int mllm_timeline_dump(unsigned long long* host, int ctas) {
  if (ctas < 1 || ctas > kCdMaxClusters * kCdCtas) return -1;
  return (int)cudaMemcpyFromSymbol(host, g_cd_tl, (size_t)ctas * kCdTlWords * sizeof(unsigned long long));
}
#endif

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

// One launch of args.nc clusters; with several clusters the launch is cooperative, so that either all
// of them are resident together or the launch fails (a cluster waits on the others' words).
cudaError_t cd_launch(const CdArgs& args, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCdCtas * args.nc);
  cfg.blockDim = dim3(kCdThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = kCdCtas;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = args.nc > 1 ? 2 : 1;
  void* params[] = {const_cast<CdArgs*>(&args)};
  return cudaLaunchKernelExC(&cfg, (const void*)cdec_kernel, params);
}

}  // namespace mllm
