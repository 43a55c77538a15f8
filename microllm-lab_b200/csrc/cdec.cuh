// Cluster decode: the single-token greedy decode loop (engine/infer.js:579-601 per token,
// engine/infer.js:625-639 for the loop) as one 16-CTA thread-block cluster per kv head (the attention
// clusters) plus helper clusters that share the MLP and lm_head rows; the clusters exchange stage
// outputs through distributed shared memory inside a cluster and through tagged global words between
// clusters.
//
// Shared by the host runtime (weight repacking, shared-memory sizing) and the kernel (cdec.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "engine.cuh"

namespace mllm {

constexpr int kCdCtas = 16;                 // CTAs of a cluster (one per SM)
constexpr int kCdMaxClusters = 8;           // clusters of one launch (kv heads + helpers)
constexpr int kCdWarps = 16;                // warps per CTA
constexpr int kCdThreads = kCdWarps * 32;   // 512
constexpr int kCdRecBytes = 320;            // one weight record: 16 rows x 32-wide group (256 B) + 16 scales
constexpr int kCdRpc = 8;                   // records per warp in one chunk of a CTA's weight stream
constexpr int kCdChunk = kCdWarps * kCdRpc * kCdRecBytes;  // 40,960 bytes: one bulk copy
constexpr int kCdMaxSlots = 4;              // chunks in flight per CTA (ring slots)
constexpr int kCdKvStage = 32;              // cache rows (K and V each) of a CTA's positions staged in shared memory
constexpr int kCdPartWords = 68;            // attention partial of one head: max, sum, 2 pad, 64 outputs
constexpr int kCdShapeError = 3;            // error flag value: the launch's cluster shape is not the packed one

// Work of one CTA in one matrix-vector stage, and its warp split.  The CTA takes the unit tiles
// [t0, t0 + T) of the stage's tile list (16 rows each) over G groups of 32 columns starting at group
// k0.  A paired stage (w1 with w3) interleaves the two matrices' tiles: unit tile 2i is w1 tile t0 + i,
// 2i + 1 is w3 tile t0 + i.  The N = Tu x G units (unit tile, group), tile-major, are dealt to the
// warps as contiguous ranges: virtual warp v takes [v q + min(v, rem), (v + 1) q + min(v + 1, rem))
// with q = N / 16, rem = N % 16.  Warp w plays virtual warp (w - off) mod 16, where off rotates by each
// stage's rem, so the extra units go round-robin and no warp's stream position drifts more than one
// record from another's.  A tile spanned by several warps gets one partial per warp, summed in warp
// order (maxc = the most per tile); a stage of one group per tile instead keeps the partials of the
// four lanes that share a row (maxc = 4).
struct CdGeom {
  int t0, T, Tu, G, k0, N, q, rem, maxc;
  int kh;  // 1: tile t0 + t covers groups [(t0 + t) % 2 G, + G) of the rows of tile (t0 + t) / 2 (K halves)
};

__host__ __device__ inline int cd_ustart(const CdGeom& g, int v) { return v * g.q + (v < g.rem ? v : g.rem); }
__host__ __device__ inline int cd_vwarp(const CdGeom& g, int u) {  // virtual warp holding unit u
  const int big = g.rem * (g.q + 1);
  return u < big ? u / (g.q + 1) : g.rem + (u - big) / (g.q > 0 ? g.q : 1);
}

__host__ __device__ inline CdGeom cd_geom(int t0, int T, int G, int k0, bool paired) {
  CdGeom g;
  g.t0 = t0;
  g.kh = 0;
  g.T = T;
  g.Tu = paired ? 2 * T : T;
  g.G = G;
  g.k0 = k0;
  g.N = g.Tu * g.G;
  g.q = g.N / kCdWarps;
  g.rem = g.N % kCdWarps;
  g.maxc = 1;
  for (int t = 0; t < g.Tu && g.G > 0; ++t) {
    const int n = cd_vwarp(g, t * g.G + g.G - 1) - cd_vwarp(g, t * g.G) + 1;
    g.maxc = g.maxc > n ? g.maxc : n;
  }
  if (g.G == 1) g.maxc = 4;  // one-group tiles keep the four lane-quad partials of each row (see run_units)
  return g;
}

// Stage kinds in stream order within a layer, then the lm_head.
//   CD_QKV:  attention cluster g (kv head g, g < nKvHeads) computes the rows of its group: q heads
//            g rep .. g rep + rep - 1, then k head g, then v head g ((rep + 2) x 64 rows); each group-local
//            tile is cut into its two K halves and the 2 (rep + 2) 4 halves are split over the 16 CTAs
//            (two partial vectors).  Helper clusters have none.
//   CD_PROJ: attention cluster g multiplies its heads' attention output (columns g rep 64 .. + rep 64
//            of proj) into a partial of all D rows; the D / 16 row tiles are split over its 16 CTAs.
//   CD_W13:  the FF rows, in slices of 16 (one w1 and one w3 tile), split over all 16 nc CTAs.
//   CD_W2:   every CTA multiplies its own h slice (the columns of its w13 rows) into a partial of all
//            D rows; a slice that covers half of a 32-column group leaves the other half of its records
//            at weight 0 (nibble 8).
//   CD_LM:   the vocab rows split over all CTAs.
enum CdStage { CD_QKV = 0, CD_PROJ = 1, CD_W13 = 2, CD_W2 = 3, CD_LM = 4 };

// FF slices (16 rows each) [s0, s1) of CTA gc of nct: its w1/w3 tiles and the h columns of its w2 records.
__host__ __device__ inline void cd_ff_slices(const ModelDev& m, int gc, int nct, int* s0, int* s1) {
  const int NS = m.FF / 16;
  *s0 = gc * NS / nct;
  *s1 = (gc + 1) * NS / nct;
}

__host__ __device__ inline CdGeom cd_stage_geom(const ModelDev& m, int st, int cid, int c, int nc) {
  const int rep = m.NH / m.NKV, nct = nc * kCdCtas, gc = cid * kCdCtas + c;
  int s0, s1;
  cd_ff_slices(m, gc, nct, &s0, &s1);
  if ((st == CD_QKV || st == CD_PROJ) && cid >= m.NKV) return cd_geom(0, 0, 2, 0, false);  // helper cluster
  switch (st) {
    case CD_QKV: {  // K halves of the group's (rep + 2) 4 tiles, so that 16 CTAs share them evenly
      const int NT = 2 * (rep + 2) * 4;
      const int t0 = c * NT / kCdCtas;
      CdGeom g = cd_geom(t0, (c + 1) * NT / kCdCtas - t0, m.D / 64, 0, false);
      g.kh = 1;
      return g;
    }
    case CD_PROJ: {
      const int NT = m.D / 16;
      const int t0 = c * NT / kCdCtas;
      return cd_geom(t0, (c + 1) * NT / kCdCtas - t0, 2 * rep, cid * 2 * rep, false);
    }
    case CD_W13: return cd_geom(s0, s1 - s0, m.D / 32, 0, true);
    case CD_W2: return s1 > s0 ? cd_geom(0, m.D / 16, (s1 + 1) / 2 - s0 / 2, s0 / 2, false)
                               : cd_geom(0, m.D / 16, 0, 0, false);
    default: {
      const int NT = (m.vocab + 15) / 16;
      const int t0 = gc * NT / nct;
      return cd_geom(t0, (gc + 1) * NT / nct - t0, m.D / 32, 0, false);
    }
  }
}

// Row of the QKV matrix at the start of group-local tile j of kv group g.
__host__ __device__ inline int cd_qkv_row(const ModelDev& m, int g, int j) {
  const int rep = m.NH / m.NKV;
  if (j < rep * 4) return g * rep * 64 + 16 * j;
  if (j < rep * 4 + 4) return m.D + g * 64 + 16 * (j - rep * 4);
  return m.D + m.NKV * 64 + g * 64 + 16 * (j - rep * 4 - 4);
}

// Rotation offset of stage `st` (CD_QKV .. CD_W2 of layer l, or CD_LM) of CTA (cid, c): the sum of
// the rems of the stages before it in the token's stream, mod 16.
__host__ __device__ inline int cd_stage_off(const ModelDev& m, int cid, int c, int nc, int l, int st) {
  int rl = 0, pre = 0;
  for (int s = CD_QKV; s <= CD_W2; ++s) {
    const int r = cd_stage_geom(m, s, cid, c, nc).rem;
    rl += r;
    if (s < st) pre += r;
  }
  if (st == CD_LM) return (m.n_layers * rl) % kCdWarps;
  return (l * rl + pre) % kCdWarps;
}

// Shared-memory plan of the kernel (byte offsets; every region 16-byte aligned).
struct CdSmem {
  int ring, actp, red, xb2, xb1, pp1, pp2, rs, qkv, attb, cand, outv, wpart, qk, mw, kvst, norms, misc, bars, feed,
      geo, total;
  int red_floats, nslot;
};

__host__ __device__ inline int cd_align16(int b) { return (b + 15) & ~15; }

// `cap`: the shared-memory limit; the ring takes as many chunk slots (up to kCdMaxSlots) as fit.
__host__ __device__ inline CdSmem cd_smem(const ModelDev& m, int cap, int nc) {
  CdSmem s;
  const int rep = m.NH / m.NKV;
  int redf = 16, outf = m.D > rep * kCdPartWords ? m.D : rep * kCdPartWords, actf = m.D;
  for (int st = 0; st <= CD_LM; ++st)
    for (int cid = 0; cid < nc; ++cid)
      for (int c = 0; c < kCdCtas; ++c) {
        const CdGeom g = cd_stage_geom(m, st, cid, c, nc);
        redf = redf > g.Tu * g.maxc * 16 ? redf : g.Tu * g.maxc * 16;
        if (st != CD_LM) outf = outf > g.T * 16 ? outf : g.T * 16;
        if (st == CD_W2) actf = actf > 32 * g.G ? actf : 32 * g.G;
      }
  int o = 0;
  auto take = [&](int bytes) {
    const int at = o;
    o += cd_align16(bytes);
    return at;
  };
  s.actp = take(actf * 4);
  s.red = take(redf * 4);
  s.xb2 = take((m.D + m.D / 4) * 4);
  s.xb1 = take((m.D + m.D / 4) * 4);
  s.pp1 = take(m.NKV * m.D * 4);          // proj partials of the attention clusters
  s.pp2 = take(nc * m.D * 4);             // w2 partials of every cluster
  s.rs = take(m.D * 4);                   // w2 partials of this CTA's D / 16 rows from the 16 CTAs
  s.qkv = take(2 * (rep + 2) * 64 * 4);  // the two K-half partials of the group's q/k/v
  s.attb = take(kCdCtas * rep * kCdPartWords * 4);
  s.cand = take(nc * kCdCtas * 16);
  s.outv = take(outf * 4);                // a stage's output rows before the push, or the attention partial
  s.wpart = take(kCdWarps * rep * kCdPartWords * 4);
  s.qk = take((rep + 2) * 64 * 4);
  s.mw = take((rep + 4) * kCdCtas * 4);   // merge weights [head][split], attention warp weights [head][warp]
  s.kvst = take(2 * kCdKvStage * 64 * 4); // staged K rows, then V rows
  s.norms = take((2 * m.n_layers + 1) * 8);
  s.misc = take(64 * 4);
  s.bars = take(16 * 8);                  // exchange barriers, the K/V staging barrier (6), one per ring slot (8 + s)
  s.feed = take(4 * kCdMaxSlots * 4);     // per slot: release count, last chunk issued
  s.geo = take(2048);                     // per stage: CdGeom, rotation offset, warp unit ranges
  o = (o + 127) & ~127;
  s.nslot = (cap - o) / kCdChunk;
  if (s.nslot > kCdMaxSlots) s.nslot = kCdMaxSlots;
  s.ring = o;
  o += s.nslot * kCdChunk;
  s.total = o;
  s.red_floats = redf;
  return s;
}

// Global exchange words between clusters, 8-byte {tag, value}, each buffer [2 parities][words]:
// proj partials [nKvHeads][D], w2 partials [nc][D], argmax candidates [16 nc][2].
enum { CD_GX_PP1 = 0, CD_GX_PP2 = 1, CD_GX_CAND = 2 };
__host__ __device__ inline size_t cd_gx_words(const ModelDev& m, int nc, int b /* -1: total */) {
  const size_t w[3] = {(size_t)m.NKV * m.D, (size_t)nc * m.D, (size_t)2 * nc * kCdCtas};
  size_t off = 0;
  for (int i = 0; i < 3; ++i) {
    if (i == b) return off;
    off += 2 * w[i];
  }
  return off;
}

// A CTA's weight stream is cpt[c] chunks per token; chunk j holds, for every warp w, its records
// [j kCdRpc, (j + 1) kCdRpc) (zero records past the warp's count).  One bulk copy moves a chunk.
struct CdArgs {
  RunArgs r;
  const uint8_t* wst;    // packed chunks of every CTA
  const uint32_t* woff;  // [16 nc] first chunk of each CTA's stream
  const uint32_t* wcpt;  // [16 nc] chunks per token of each CTA
  const uint32_t* wcnt;  // [16 nc x kCdWarps] records per token of each warp
  CdSmem L;              // shared-memory plan (cd_smem)
  int nc;                // clusters of the launch: nKvHeads attention clusters, then helpers
  uint64_t* gx;          // global exchange words (cd_gx_words), zeroed before the first launch; null if nc = 1
  uint32_t tag0;         // tags of this launch are tag0 + 1 + use index (uses < 2^22 per launch)
};

// ---- host side (cdec.cu)

// One Q4 matrix in host memory (PGW layout).
struct HostQ4 {
  const uint8_t* w;
  const uint8_t* s;  // f32 scales, possibly unaligned
  int rows, K;
};

bool cd_supported(const ModelDev& m, size_t smem_cap, int nc);
size_t cd_smem_bytes(const ModelDev& m, size_t smem_cap, int nc);
void cd_pack(const ModelDev& m, int nc, const std::vector<HostQ4>& mats, const HostQ4& lm, std::vector<uint8_t>* out,
             std::vector<uint32_t>* off, std::vector<uint32_t>* cpt, std::vector<uint32_t>* cnt);
cudaError_t cd_setup(size_t smem_cap);
int cd_max_clusters(size_t smem);
cudaError_t cd_launch(const CdArgs& args, size_t smem, cudaStream_t st);

}  // namespace mllm
