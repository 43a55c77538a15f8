// Device helpers shared by the decode kernels: flag-in-data exchange words, bounded waits, Q4 dequant.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace mllm {

constexpr int kThreads = 256;  // 8 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kHeadDim = 64;   // every supported model (PetitGPT, SmolLM2, GPT-2) uses 64
constexpr unsigned long long kWaitNs = 500ull * 1000 * 1000;  // default per-wait limit: 0.5 s

// ---------------------------------------------------------------------------------------------
// Exchange words.  A produced value travels with a 32-bit tag in one 8-byte word; a consumer spins
// until the tag equals the forward's tag.  8-byte aligned accesses are single-copy atomic, so no
// fence or separate flag is needed between value and tag.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t ll_load(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Two adjacent exchange words in one 16-byte load (p 16-byte aligned; each word single-copy atomic).
__device__ __forceinline__ void ll_load2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void ll_store_word(uint64_t* p, uint64_t w) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void ll_store(uint64_t* p, uint32_t tag, float v) {
  ll_store_word(p, ((uint64_t)tag << 32) | __float_as_uint(v));
}
__device__ __forceinline__ void ll_store_u32(uint64_t* p, uint32_t tag, uint32_t v) {
  ll_store_word(p, ((uint64_t)tag << 32) | v);
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait state of one CTA.  Every spin checks the clock every few rounds; when the limit passes, or
// another CTA has raised the error flag, the wait gives up and the kernel returns.
struct Waiter {
  int* err;           // device-wide error flag (0 = ok)
  uint64_t limit_ns;  // per-wait limit
  __device__ __forceinline__ bool give_up(uint64_t start) const {
    if (*(volatile int*)err) return true;
    if (globaltimer() - start > limit_ns) {
      atomicCAS(err, 0, 1);
      return true;
    }
    return false;
  }
};

// Read-only loads issued exactly where written.  The compiler treats __ldg as an invariant load that
// it may sink below a later wait; these volatile forms keep a prefetch ahead of the wait it overlaps.
__device__ __forceinline__ uint32_t ldv_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float ldv_f32(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldcg_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

// Bulk prefetch of [p, p + bytes) into L2 (no data returned to the SM).  p 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Bulk global -> shared copies (cp.async.bulk, completion counted on a CTA mbarrier).  dst and src
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Wait for phase `parity` of an mbarrier for at most limit_ns; false when the limit ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > limit_ns) return false;
  return true;
}

// Read-only load with an L2 cache policy (createpolicy); policy 0 means the default path.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint32_t ld_hint_u32(const uint32_t* ptr, uint64_t pol) {
  uint32_t v;
  asm volatile("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(ptr), "l"(pol));
  return v;
}

// ---------------------------------------------------------------------------------------------
// Q4 group-32 dequant.  A u32 word of a packed row holds 8 consecutive elements: byte b carries
// element 2b in its low nibble and 2b+1 in its high nibble (tools/convert_hf_to_pgw.py:33).
// (q - 8) is produced exactly in fp32 from the bit pattern 0x4B000000 | q (= 2^23 + q).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float nib_at(uint32_t bytes4, int j) {
  return __uint_as_float(__byte_perm(bytes4, 0x4B000000u, 0x7440u | (unsigned)j)) - 8388616.0f;
}

// sum_{e<8} (q_e - 8) * x[e], accumulated in element order.
__device__ __forceinline__ float word_dot(uint32_t u, const float* x) {
  const uint32_t lo = u & 0x0F0F0F0Fu, hi = (u >> 4) & 0x0F0F0F0Fu;
  const float4 xa = *reinterpret_cast<const float4*>(x);
  const float4 xb = *reinterpret_cast<const float4*>(x + 4);
  float s = nib_at(lo, 0) * xa.x;
  s = fmaf(nib_at(hi, 0), xa.y, s);
  s = fmaf(nib_at(lo, 1), xa.z, s);
  s = fmaf(nib_at(hi, 1), xa.w, s);
  s = fmaf(nib_at(lo, 2), xb.x, s);
  s = fmaf(nib_at(hi, 2), xb.y, s);
  s = fmaf(nib_at(lo, 3), xb.z, s);
  s = fmaf(nib_at(hi, 3), xb.w, s);
  return s;
}

// ---------------------------------------------------------------------------------------------
// Token streaming into mapped host memory: word 0 counts the ids published, ids follow from word
// kStreamHead (bits 30-31 carry the phase: 0 prefill, 1 decode, 2 accepted draft).  The id is stored
// first and the count with a system-scope release, so a host thread that reads the count sees every
// id below it.
// ---------------------------------------------------------------------------------------------
constexpr int kStreamHead = 16;
__device__ __forceinline__ void stream_publish(int32_t* s, int i, int id, int phase) {
  if (!s) return;
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(s + kStreamHead + i), "r"(id | (phase << 30)) : "memory");
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(s), "r"(i + 1) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mllm
