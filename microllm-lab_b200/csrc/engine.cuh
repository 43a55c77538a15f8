// Device-side descriptors shared by the host runtime (engine.cu) and the decode kernel (decode.cu).
#pragma once
#include <cstdint>

namespace mllm {

// One Q4 matrix in the PGW layout: `w` = packed rows as u32 words ([rows][cols/8]),
// `s` = f32 scales ([rows][cols/32]).
struct Q4 {
  const uint32_t* w;
  const float* s;
};

struct LayerDev {
  Q4 qkv, proj, w1, w3, w2;  // GPT-2: w1 = mlp.fc, w2 = mlp.proj, w3 unused
  const float* norm1;        // llama: gain [D]; GPT-2: ln1 [gain; bias] (2D)
  const float* norm2;
  const float* qkv_b;        // GPT-2 biases (null for llama)
  const float* proj_b;
  const float* fc_b;
  const float* mproj_b;
};

struct ModelDev {
  int arch;  // 0 llama, 1 gpt2
  int vocab, n_layers, D, NH, NKV, FF, QKV, max_seq, kv_len, rope_dim;
  const LayerDev* layers;  // device array [n_layers]
  Q4 lm;                   // tied lm_head, also the token embedding (engine/infer.js:360-420)
  const float* norm_f;     // llama norm_f [D]; GPT-2 ln_f [2D]
  const float* wpe;        // GPT-2 [max_seq][D]
  const float* sf;         // GPT-2 scale_factors [D] (null when absent)
  const float* rope_cos;   // [max_seq][rope_dim] (engine/infer.js:185-206)
  const float* rope_sin;
};

// Exchange buffers (8-byte tagged words).  Each is [n_layers][mmax][stride] with strides padded to
// 32 words; `cand` is [2][grid][mmax][4].
// Single-token attention split over positions: at most kAttnSplits CTAs per head, one per kAttnRound
// positions; a split's partial is kAttnPartWords tagged words (max, sum, 2 zero, 64 outputs).
constexpr int kAttnSplits = 16;
constexpr int kAttnRound = 128;
constexpr int kAttnMinRounds = 3;
constexpr int kAttnPartWords = 68;
// Partials of the single-token attention splits: [layers][NH][kAttnSplits][kAttnPartWords] words
// placed right after the argmax candidate words (2 x grid x mmax x 4) in the same allocation.
inline __host__ __device__ size_t attn_partials_offset(int grid, int mmax) { return (size_t)2 * grid * mmax * 4; }
inline __host__ __device__ size_t attn_partials_words(int layers, int nh) {
  return (size_t)layers * nh * kAttnSplits * kAttnPartWords;
}

struct ExchangeDev {
  uint64_t* qkv;
  uint64_t* att;
  uint64_t* x1;
  uint64_t* a;
  uint64_t* x2;
  uint64_t* cand;  // argmax candidates, then the single-token attention partials (attn_partials_offset)
  int s_qkv, s_d, s_ff;  // row strides in words
};

enum RunMode { MODE_FORWARD = 0, MODE_GENERATE = 1, MODE_SELFTEST_WAIT = 2 };

// Status words written by CTA 0 (int32 view): see the layout in engine.cu.
enum StatusIdx {
  ST_NGEN = 0,
  ST_STOP = 1,
  ST_HITS = 2,
  ST_TRIES = 3,
  ST_FORWARDS = 4,
  ST_ERR = 5,
  ST_T0 = 6,      // u64 globaltimer at kernel start (2 words)
  ST_TFIRST = 8,  // u64 at the first generated id
  ST_TEND = 10,   // u64 at the end
  ST_WORDS = 16
};

struct RunArgs {
  ModelDev m;
  ExchangeDev x;
  float* kc;  // slot K cache [n_layers][NKV][kv_len][64]
  float* vc;
  int mmax;   // token rows per layer in the exchange buffers (tokens per forward of the general kernel)
  int srows;  // token rows held in shared memory: mmax for the general kernel, 1 for the single-token one
  int mode;
  // request
  const int32_t* ids;  // device prompt / forward ids
  int n_ids;
  int pos0;            // MODE_FORWARD: position of ids[0]
  int logits_each;     // MODE_FORWARD
  float* logits;       // MODE_FORWARD, nullable: [rows][vocab]
  int32_t* argmax_out; // MODE_FORWARD, nullable
  int max_new;         // MODE_GENERATE
  int eos;
  int spec_k;
  int ngram;
  int32_t* out_ids;    // MODE_GENERATE: [max_new]
  int32_t* stream_ids; // MODE_GENERATE, nullable: mapped host words the ids are also published to
  int32_t* status;     // [ST_WORDS]
  uint32_t base_tag;
  int* err;
  uint64_t wait_ns;    // per-wait limit (0 = kWaitNs)
  int start_gen;       // MODE_GENERATE: ids already generated (in out_ids) by an earlier launch; 0 = prefill first
  int prefill_only;    // MODE_GENERATE: stop after the first generated id
  int poll_sleep_ns;   // back-off between unsuccessful poll rounds (0 = spin)
  int weight_policy;   // 0: default L2 policy for weights, 1: evict_last
  int l2_prefetch;     // 1: bulk-prefetch the next layer's weight slices (and the layer's K/V) into L2
  int lm_rpc;          // single-token kernel: > 0 = each CTA keeps lm_head rows [cta * lm_rpc, +lm_rpc) in
                       // shared memory for the whole launch (copied once at entry)
};

}  // namespace mllm
