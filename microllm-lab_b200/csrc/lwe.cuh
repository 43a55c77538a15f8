// Arguments of the layer-wise engine kernels (lwe.cu), shared with the host runtime (engine.cu).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>
#include <vector>

#include "engine.cuh"

namespace mllm {

constexpr int kLweMaxRep = 4;  // query heads per kv head handled by one attention CTA
constexpr int kLweSsStride = 16;  // per-token partial sums of squares: one per 64-row tile of dModel <= 1024

struct LweArgs {
  ModelDev m;
  int layer;
  float* x;               // [tmax][D] residual stream
  __half* xh;             // [tmax][ldx] fp16 hi of the GEMM input (norm / attention output)
  __half* xl;
  int ldx;
  __half* xh2;            // [tmax][ldx2] fp16 hi of the w2 / mlp.proj input
  __half* xl2;
  int ldx2;
  __half* xh3;            // [tmax][ldx] fp16 hi of norm2 output when RMSNorm is folded into the GEMMs
  __half* xl3;
  float* ss;              // [tmax][kLweSsStride] partial sums of squares of x per 64-row tile
  int fold;               // RMSNorm folded into the GEMMs for this forward
  int tiled;              // the forward's GEMMs run on the tcgen05 tile: xh/xl, xh2/xl2 and xh3/xl3 hold
                          // the tiled layout (tc5::tiled_at) instead of [tmax][ld] rows
  float* qkv;             // [tmax][QKV]
  int32_t* tok;           // [tmax] token ids
  int32_t* slot;          // [tmax] sequence slots
  int32_t* pos;           // [tmax] positions
  float* const* kc;       // [max_slots] per-slot K cache bases ([layer][kvHead][kvLen][64])
  float* const* vc;
  float* pval;            // [nblk][lm_cap] lm_head argmax partials
  int32_t* pidx;
  int lm_cap;
  int32_t* amax;          // [lm_cap] argmax per lm row
  int32_t* lm_src;        // [lm_cap] token index of each lm row
  int* err;               // device error flag: 2 = a token id out of range
  const int* skip;        // when set and *skip != 0 every kernel of the forward returns at once
  float* skws;            // split-K partial tiles [kLweSkwsBytes]
  int* skctr;             // [kLweSplitKTiles] zeroed split-K tile counters
};
constexpr size_t kLweSplitKBytes = size_t(8) << 20;   // split-K partials of the mma.sync GEMMs
constexpr size_t kLweSkwsBytes = size_t(32) << 20;    // the workspace (the tcgen05 GEMMs use all of it)
constexpr int kLmWideRows = 64;  // lm rows from which the persistent lm_head GEMM is used
constexpr int kW13WideRows = 512;  // token rows from which the persistent w1/w3 GEMM is used
constexpr int kLweSplitAttnRows = 16;  // forwards of at most this many tokens use the position-split attention
constexpr int kLweSplitKTiles = 16384;
constexpr int kTc5GemmRows = 32;  // token rows from which the layer GEMMs run on the tcgen05 tile

// A layer matrix expanded once at load into the tcgen05 tile's group images (tc5::tc5_expand_kernel):
// img [row tiles][groups][16 KB], down [row tiles] (each tile's 2^-E).
struct Tc5Pre {
  uint8_t* img = nullptr;
  float* down = nullptr;
};
enum { kPreQkv = 0, kPreProj = 1, kPreW13 = 2, kPreW2 = 3, kPreMats = 4 };
// Row tiles and bytes of one matrix's images (paired: w1/w3 interleaved, 64 FF rows a tile).
int tc5_pre_tiles(int R, bool paired);
size_t tc5_pre_bytes(int R, int K, bool paired);
cudaError_t tc5_expand(const Q4& w, const Q4* w3, int R, int K, const Tc5Pre& p, cudaStream_t st);

// Host-side copies of the per-layer descriptors the launches pass by value.
struct LweHost {
  std::vector<LayerDev> layers;
  float* attn_part = nullptr;  // [tmax][NKV][splits][rep][66] decode-attention partials
  int* attn_ctr = nullptr;     // [tmax * NKV] zeroed split counters
  size_t attn_ctr_n = 0;
  int attn_split = 0;  // decode attention split over positions (MLLM_LWE_ATTN_SPLIT=1)
  int fold_norm = 1;   // llama RMSNorm folded into the GEMM epilogues (MLLM_LWE_FOLD_NORM=0: norm kernels)
  int pdl = 1;         // programmatic dependent launch between the forward's kernels (MLLM_LWE_PDL=0: off)
  int lm_wide = 1;     // persistent lm_head GEMM for many rows without logits (MLLM_LWE_LM_WIDE=0: off)
  int lm_tc5 = 1;      // the same on the tcgen05 tile, ahead of lm_wide (MLLM_LWE_LM_TC5=0: off)
  std::vector<Tc5Pre> pre;  // [layer * kPreMats + matrix] when the layer GEMMs run on the tcgen05 tile
  int gemm_tc5 = 0;    // llama forwards of >= kTc5GemmRows rows: every layer GEMM on the tcgen05 tile
                       // (MLLM_LWE_GEMM_TC5=1; off by default: measured slower than the mma.sync tiles
                       // at these shapes)
  int w13_wide = 1;    // persistent w1/w3 GEMM for long forwards (MLLM_LWE_W13_WIDE=0: off)
  int rope_epi = 1;    // RoPE + K/V cache rows in the QKV GEMM epilogue (MLLM_LWE_ROPE_EPI=0: lwe_rope_kv)
};

// one_per_slot: every token belongs to a different slot (a batched decode step), which lets the
// attention kernel apply RoPE and write the K/V row itself.
cudaError_t lwe_forward(LweArgs a, const LweHost& h, int T, int lm_T, bool lm_from_src, float* logits,
                        bool one_per_slot, cudaStream_t st);
// Positions per split and split count of the decode-step attention for a cache of kv_len positions.
void lwe_attn_split_shape(int kv_len, int* chunk, int* splits);
// One-time function attributes (call once per device before the first forward).
cudaError_t lwe_setup(int kv_len);
// One prompt (or forward) chunk of a single slot: ids (device) at positions pos0.., lm rows either
// every token (lm_each) or the last one.
void lwe_fill(LweArgs a, const int32_t* ids, int n, int slot, int pos0, int lm_each, cudaStream_t st);
void lwe_first(LweArgs a, int32_t* out_ids, int32_t* status, int eos, int forwards, int32_t* stream, cudaStream_t st);
void lwe_mark_time(int32_t* status, int idx, cudaStream_t st);
// Prompt-lookup speculation: device loop state (int32 words), draft [kSpecDraft, +16) and history
// [kSpecHist, +kv_len + 64).  The done word is SpecWord 3.
constexpr int kSpecDraft = 16;
constexpr int kSpecHist = 64;
constexpr int kSpecMaxK = 15;
constexpr int kSpecDoneWord = 3;
void lwe_spec_init(int32_t* sp, const int32_t* ids, int n, const int32_t* out_ids, int max_new, int eos, int kv_len,
                   int prefill_forwards, cudaStream_t st);
cudaError_t lwe_spec_iteration(LweArgs a, const LweHost& h, int32_t* sp, int32_t* out_ids, int spec_k, int ngram,
                               int max_new, int eos, int slot, int32_t* stream, cudaStream_t st);
void lwe_spec_finish(const int32_t* sp, int32_t* status, cudaStream_t st);
// Kernel launches issued so far by the calling thread through these functions.
long lwe_launch_count();
// Replicated multi-sequence decode
void lwe_gather(int32_t* tok, const int32_t* ids, const int32_t* src, int n, cudaStream_t st);
void lwe_batch_first(const int32_t* amax, const int32_t* lm_slot, int nlm, int max_new, int eos, int kv_len,
                     int32_t* out_ids, int32_t* counts, const int32_t* lens, cudaStream_t st);
void lwe_batch_decode_setup(LweArgs a, int n, const int32_t* out_ids, const int32_t* counts, const int32_t* lens,
                            int max_new, cudaStream_t st);
void lwe_batch_advance(LweArgs a, int n, int max_new, int eos, int32_t* out_ids, int32_t* counts,
                       const int32_t* lens, cudaStream_t st);
void lwe_count_active(const int32_t* counts, int n, int32_t* active, cudaStream_t st);
size_t lwe_argmax_pen_smem(int V, int max_new);
void lwe_penalised_argmax(const float* logits, int V, int T, const int32_t* out_ids, const int32_t* counts, int max_new,
                          int32_t* amax, cudaStream_t st);

}  // namespace mllm
