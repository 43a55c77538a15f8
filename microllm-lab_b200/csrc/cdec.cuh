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
constexpr int kCdRing = 24;                 // records in each warp's private ring
constexpr int kCdBatch = 4;                 // records per cp.async group
constexpr int kCdKvPre = 4;                 // K/V positions per warp held in registers ahead of attention
constexpr int kCdPartWords = 68;            // attention partial of one head: max, sum, 2 pad, 64 outputs

// Row split of one matrix-vector stage for one CTA, and its warp split.  The stage's rows form
// NT = ceil(rows / 16) tiles; CTA c takes tiles [t0, t0 + T).  A paired stage (w1 with w3) interleaves
// the two matrices' tiles: unit tile 2i is w1 tile t0 + i, 2i + 1 is w3 tile t0 + i.  The CTA's Tu unit
// tiles x G groups of 32 are split over the 16 warps as KW k-slices x TW tile sets (KW x TW = 16):
// warp w takes groups [ks G / KW, (ks + 1) G / KW) (ks = w % KW) of unit tiles w / KW, w / KW + TW, ...
// KW is the power of two that minimises the largest warp's record count (ties: the smaller KW).
struct CdGeom {
  int t0, T, Tu, G, KW, TW;
};

__host__ __device__ inline CdGeom cd_geom(int rows, int K, bool paired, int c) {
  const int NT = (rows + 15) / 16;
  CdGeom g;
  g.t0 = (c * NT) / kCdCtas;
  g.T = ((c + 1) * NT) / kCdCtas - g.t0;
  g.Tu = paired ? 2 * g.T : g.T;
  g.G = K / 32;
  int best = 1 << 30, bk = 1;
  for (int kw = 1; kw <= kCdWarps; kw *= 2) {
    const int tw = kCdWarps / kw;
    const int u = ((g.Tu + tw - 1) / tw) * ((g.G + kw - 1) / kw);
    if (u < best) {
      best = u;
      bk = kw;
    }
  }
  g.KW = bk;
  g.TW = kCdWarps / bk;
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

// Attention work: NKV x S units (kv head, split of positions), S = max(1, 16 / NKV); unit u runs on
// CTA u.
__host__ __device__ inline int cd_splits(const ModelDev& m) { return m.NKV >= kCdCtas ? 1 : kCdCtas / m.NKV; }

// Shared-memory plan of the kernel (byte offsets; every region 16-byte aligned).
struct CdSmem {
  int ring, actp, red, xb2, xb1, qkv, hb, attb, cand, outv, wpart, qk, mw, norms, misc, bars, total;
  int red_floats;
};

__host__ __device__ inline int cd_align16(int b) { return (b + 15) & ~15; }

__host__ __device__ inline CdSmem cd_smem(const ModelDev& m) {
  CdSmem s;
  const int rep = m.NH / m.NKV;
  int redf = 16;
  for (int st = 0; st <= CD_LM; ++st) {
    int rows, K;
    bool paired;
    cd_stage_shape(m, st, &rows, &K, &paired);
    for (int c = 0; c < kCdCtas; ++c) {
      const CdGeom g = cd_geom(rows, K, paired, c);
      redf = redf > g.Tu * g.KW * 16 ? redf : g.Tu * g.KW * 16;
    }
  }
  int o = 0;
  auto take = [&](int bytes) {
    const int at = o;
    o += cd_align16(bytes);
    return at;
  };
  s.ring = take(kCdWarps * kCdRing * kCdRecBytes);
  s.actp = take((m.FF > m.D ? m.FF : m.D) * 4);
  s.red = take(redf * 4);
  s.xb2 = take((m.D + m.D / 4) * 4);
  s.xb1 = take((m.D + m.D / 4) * 4);
  s.qkv = take(m.QKV * 4);
  s.hb = take(m.FF * 4);
  s.attb = take(kCdCtas * rep * kCdPartWords * 4);
  s.cand = take(kCdCtas * 16);
  s.outv = take(rep * kCdPartWords * 4);
  s.wpart = take(kCdWarps * rep * kCdPartWords * 4);
  s.qk = take((rep + 2) * 64 * 4);
  s.mw = take((m.NH + 4) * kCdCtas * 4);  // merge weights [head][split], attention warp weights [head][warp]
  s.norms = take((2 * m.n_layers + 1) * 8);
  s.misc = take(64 * 4);
  s.bars = take(8 * 8);
  s.total = o;
  s.red_floats = redf;
  return s;
}

struct CdArgs {
  RunArgs r;
  const uint4* wst;      // packed weight records of every warp's stream
  const uint32_t* woff;  // [kCdCtas * kCdWarps] first record of each warp's stream
  const uint32_t* wcnt;  // [kCdCtas * kCdWarps] records per token of each warp's stream
};

// ---- host side (cdec.cu)

// One Q4 matrix in host memory (PGW layout).
struct HostQ4 {
  const uint8_t* w;
  const uint8_t* s;  // f32 scales, possibly unaligned
  int rows, K;
};

bool cd_supported(const ModelDev& m, size_t smem_cap);
size_t cd_smem_bytes(const ModelDev& m);
void cd_pack(const ModelDev& m, const std::vector<HostQ4>& mats, const HostQ4& lm, std::vector<uint8_t>* out,
             std::vector<uint32_t>* off, std::vector<uint32_t>* cnt);
cudaError_t cd_setup(size_t smem_cap);
int cd_max_clusters(size_t smem);
cudaError_t cd_launch(const CdArgs& args, size_t smem, cudaStream_t st);

}  // namespace mllm
