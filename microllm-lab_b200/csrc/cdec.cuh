// Cluster decode: the single-token greedy decode loop (engine/infer.js:579-601 per token,
// engine/infer.js:625-639 for the loop) as ONE thread-block cluster of 16 CTAs that exchange every
// stage output through distributed shared memory.
//
// Shared by the host runtime (weight repacking, shared-memory sizing) and the kernel (cdec.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "engine.cuh"

namespace mllm {

constexpr int kCdCtas = 16;                 // CTAs of the cluster (one per SM)
constexpr int kCdWarps = 16;                // warps per CTA
constexpr int kCdThreads = kCdWarps * 32;   // 512
constexpr int kCdRecBytes = 320;            // one weight record: 16 rows x 32-wide group (256 B) + 16 scales
constexpr int kCdRpc = 8;                   // records per warp in one chunk of a CTA's weight stream
constexpr int kCdChunk = kCdWarps * kCdRpc * kCdRecBytes;  // 40,960 bytes: one bulk copy
constexpr int kCdMaxSlots = 4;              // chunks in flight per CTA (ring slots)
constexpr int kCdKvPre = 4;                 // K/V positions per warp held in registers ahead of attention
constexpr int kCdPartWords = 68;            // attention partial of one head: max, sum, 2 pad, 64 outputs

// Row split of one matrix-vector stage for one CTA, and its warp split.  The stage's rows form
// NT = ceil(rows / 16) tiles; CTA c takes tiles [t0, t0 + T).  A paired stage (w1 with w3) interleaves
// the two matrices' tiles: unit tile 2i is w1 tile t0 + i, 2i + 1 is w3 tile t0 + i.  The CTA's
// N = Tu x G units (unit tile, group of 32), tile-major, are dealt to the warps as contiguous ranges:
// virtual warp v takes [v q + min(v, rem), (v + 1) q + min(v + 1, rem)) with q = N / 16, rem = N % 16.
// Warp w plays virtual warp (w - off) mod 16, where off rotates by each stage's rem, so the extra units
// go round-robin and no warp's stream position drifts more than one record from another's.  A tile
// spanned by several warps gets one partial per warp, summed in warp order (maxc = the most per tile).
struct CdGeom {
  int t0, T, Tu, G, N, q, rem, maxc;
};

__host__ __device__ inline int cd_ustart(const CdGeom& g, int v) { return v * g.q + (v < g.rem ? v : g.rem); }
__host__ __device__ inline int cd_vwarp(const CdGeom& g, int u) {  // virtual warp holding unit u
  const int big = g.rem * (g.q + 1);
  return u < big ? u / (g.q + 1) : g.rem + (u - big) / (g.q > 0 ? g.q : 1);
}

__host__ __device__ inline CdGeom cd_geom(int rows, int K, bool paired, int c) {
  const int NT = (rows + 15) / 16;
  CdGeom g;
  g.t0 = (c * NT) / kCdCtas;
  g.T = ((c + 1) * NT) / kCdCtas - g.t0;
  g.Tu = paired ? 2 * g.T : g.T;
  g.G = K / 32;
  g.N = g.Tu * g.G;
  g.q = g.N / kCdWarps;
  g.rem = g.N % kCdWarps;
  g.maxc = 1;
  for (int t = 0; t < g.Tu; ++t) {
    const int n = cd_vwarp(g, t * g.G + g.G - 1) - cd_vwarp(g, t * g.G) + 1;
    g.maxc = g.maxc > n ? g.maxc : n;
  }
  return g;
}

// Stage kinds in stream order within a layer, then the lm_head.
enum CdStage { CD_QKV = 0, CD_PROJ = 1, CD_W13 = 2, CD_W2 = 3, CD_LM = 4 };

__host__ __device__ inline void cd_stage_shape(const ModelDev& m, int s, int* rows, int* K, bool* paired) {
  *paired = s == CD_W13;
  switch (s) {
    case CD_QKV: *rows = m.QKV; *K = m.D; break;
    case CD_PROJ: *rows = m.D; *K = m.D; break;
    case CD_W13: *rows = m.FF; *K = m.D; break;
    case CD_W2: *rows = m.D; *K = m.FF; break;
    default: *rows = m.vocab; *K = m.D; break;
  }
}

// Rotation offset of stage `st` (CD_QKV .. CD_W2 of layer l, or CD_LM) of CTA c: the sum of the
// rems of the stages before it in the token's stream, mod 16.
__host__ __device__ inline int cd_stage_off(const ModelDev& m, int c, int l, int st);

// Attention work: NKV x S units (kv head, split of positions), S = max(1, 16 / NKV); unit u runs on
// CTA u.
__host__ __device__ inline int cd_splits(const ModelDev& m) { return m.NKV >= kCdCtas ? 1 : kCdCtas / m.NKV; }

__host__ __device__ inline int cd_stage_off(const ModelDev& m, int c, int l, int st) {
  int rl = 0, pre = 0;
  for (int s = CD_QKV; s <= CD_W2; ++s) {
    int rows, K;
    bool paired;
    cd_stage_shape(m, s, &rows, &K, &paired);
    const int r = cd_geom(rows, K, paired, c).rem;
    rl += r;
    if (s < st) pre += r;
  }
  if (st == CD_LM) return (m.n_layers * rl) % kCdWarps;
  return (l * rl + pre) % kCdWarps;
}

// Shared-memory plan of the kernel (byte offsets; every region 16-byte aligned).
struct CdSmem {
  int ring, actp, red, xb2, xb1, qkv, hb, attb, cand, outv, wpart, qk, mw, norms, misc, bars, feed, total;
  int red_floats, nslot;
};

__host__ __device__ inline int cd_align16(int b) { return (b + 15) & ~15; }

// `cap`: the shared-memory limit; the ring takes as many chunk slots (up to kCdMaxSlots) as fit.
__host__ __device__ inline CdSmem cd_smem(const ModelDev& m, int cap) {
  CdSmem s;
  const int rep = m.NH / m.NKV;
  int redf = 16, outf = rep * kCdPartWords;
  for (int st = 0; st <= CD_LM; ++st) {
    int rows, K;
    bool paired;
    cd_stage_shape(m, st, &rows, &K, &paired);
    for (int c = 0; c < kCdCtas; ++c) {
      const CdGeom g = cd_geom(rows, K, paired, c);
      redf = redf > g.Tu * g.maxc * 16 ? redf : g.Tu * g.maxc * 16;
      if (st != CD_LM) outf = outf > g.T * 16 ? outf : g.T * 16;
    }
  }
  int o = 0;
  auto take = [&](int bytes) {
    const int at = o;
    o += cd_align16(bytes);
    return at;
  };
  s.actp = take((m.FF > m.D ? m.FF : m.D) * 4);
  s.red = take(redf * 4);
  s.xb2 = take((m.D + m.D / 4) * 4);
  s.xb1 = take((m.D + m.D / 4) * 4);
  s.qkv = take(m.QKV * 4);
  s.hb = take(m.FF * 4);
  s.attb = take(kCdCtas * rep * kCdPartWords * 4);
  s.cand = take(kCdCtas * 16);
  s.outv = take(outf * 4);  // a stage's output rows before the push, or the attention partial
  s.wpart = take(kCdWarps * rep * kCdPartWords * 4);
  s.qk = take((rep + 2) * 64 * 4);
  s.mw = take((m.NH + 4) * kCdCtas * 4);  // merge weights [head][split], attention warp weights [head][warp]
  s.norms = take((2 * m.n_layers + 1) * 8);
  s.misc = take(64 * 4);
  s.bars = take(16 * 8);                  // exchange barriers, then one full barrier per ring slot
  s.feed = take(4 * kCdMaxSlots * 4);     // per slot: release count, last chunk issued
  o = (o + 127) & ~127;
  s.nslot = (cap - o) / kCdChunk;
  if (s.nslot > kCdMaxSlots) s.nslot = kCdMaxSlots;
  s.ring = o;
  o += s.nslot * kCdChunk;
  s.total = o;
  s.red_floats = redf;
  return s;
}

// A CTA's weight stream is cpt[c] chunks per token; chunk j holds, for every warp w, its records
// [j kCdRpc, (j + 1) kCdRpc) (zero records past the warp's count).  One bulk copy moves a chunk.
struct CdArgs {
  RunArgs r;
  const uint8_t* wst;    // packed chunks of every CTA
  const uint32_t* woff;  // [kCdCtas] first chunk of each CTA's stream
  const uint32_t* wcpt;  // [kCdCtas] chunks per token of each CTA
  const uint32_t* wcnt;  // [kCdCtas * kCdWarps] records per token of each warp
  int smem_cap;          // the shared-memory limit the plan (cd_smem) was made for
};

// ---- host side (cdec.cu)

// One Q4 matrix in host memory (PGW layout).
struct HostQ4 {
  const uint8_t* w;
  const uint8_t* s;  // f32 scales, possibly unaligned
  int rows, K;
};

bool cd_supported(const ModelDev& m, size_t smem_cap);
size_t cd_smem_bytes(const ModelDev& m, size_t smem_cap);
void cd_pack(const ModelDev& m, const std::vector<HostQ4>& mats, const HostQ4& lm, std::vector<uint8_t>* out,
             std::vector<uint32_t>* off, std::vector<uint32_t>* cpt, std::vector<uint32_t>* cnt);
cudaError_t cd_setup(size_t smem_cap);
int cd_max_clusters(size_t smem);
cudaError_t cd_launch(const CdArgs& args, size_t smem, cudaStream_t st);

}  // namespace mllm
