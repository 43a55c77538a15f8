// Host runtime of the B200 Q4 decode backend: the C ABI declared in include/mllm.h.
//
// mllm_create  : engine/weights.js:5-40 parsePgw + engine/infer.js:290-336 binding + GpuPetitGPT.init
//                (engine/webgpu.js:892-1106): Q4 matrices are uploaded in their PGW layout, f32 norms,
//                biases and wpe as they are; the RoPE table is built like engine/infer.js:185-206.
// mllm_forward : forwardPrompt / forwardDecode / the verify forward (engine/infer.js:553-601,
//                engine/webgpu.js:1248).
// mllm_generate: engine/infer.js:603-646 and engine/webgpu.js:1164-1282 in one device launch.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/mllm.h"
#include "cdec.cuh"
#include "device_common.cuh"
#include "engine.cuh"
#include "lwe.cuh"
#include "pgw.hpp"

namespace mllm {
size_t decode_smem_bytes(const ModelDev& md, int srows, int grid);
size_t decode1_smem_bytes(const ModelDev& md, int grid, int lm_rpc);
typedef void (*DecodeFn)(const RunArgs);
DecodeFn pick_decode_kernel(int D, int FF, bool multi);
DecodeFn pick_decode1_kernel(int D, int FF, bool split);
void set_global_error(const char* msg);
}  // namespace mllm

using namespace mllm;

namespace {

thread_local std::string g_create_error;

}  // namespace

// Message for mllm_last_error(NULL) from entry points that have no handle.
void mllm::set_global_error(const char* msg) { g_create_error = msg; }

namespace {

struct Slot {
  float* k = nullptr;
  float* v = nullptr;
  int cache_len = 0;
};

// Device buffer that grows on demand (freed and reallocated; the stream is drained first).
struct Grow {
  void* p = nullptr;
  size_t cap = 0;
};

}  // namespace

struct mllm_engine {
  int device = 0;
  PgwModel pgw;
  ModelDev md{};
  ExchangeDev ex{};
  DecodeFn kernel_multi = nullptr;   // prefill chunks, verify forwards, speculation
  DecodeFn kernel_single = nullptr;  // one token per forward: the greedy decode loop
  DecodeFn kernel_single_split = nullptr;  // the same with position-split attention (long contexts)
  int grid = 0, mmax = 0;
  size_t smem_multi = 0, smem_single = 0;
  cudaStream_t stream = nullptr;     // launches go here
  cudaStream_t own_stream = nullptr; // created with the handle
  std::vector<void*> allocs;
  size_t bytes = 0;
  std::vector<Slot> slots;
  int32_t* d_ids = nullptr;   // [kv_len + 16]
  int32_t* d_out = nullptr;   // [kv_len + 16]
  int32_t* d_status = nullptr;
  int* d_err = nullptr;
  float* d_logits = nullptr;
  size_t logits_cap = 0;      // floats
  int32_t* d_argmax = nullptr;
  int32_t* h_status = nullptr;  // pinned [ST_WORDS + 1]
  uint32_t tag = 1;
  std::string err;
  int poll_sleep_ns = 200;     // MLLM_POLL_SLEEP_NS: back-off between poll rounds (less L2 contention)
  int weight_policy = 0;       // MLLM_WEIGHT_EVICT_LAST
  int l2_prefetch = 1;         // MLLM_L2_PREFETCH (default on)
  int lm_rpc = 0;              // lm_head rows per CTA kept in the single-token kernel's shared memory
  // layer-wise engine: token-batch forwards on the tensor cores (prefill, verify, batched decode)
  int lwe_ok = 0;              // rep = nHeads / nKvHeads fits its attention kernel (else multi-token forwards
                               // run on the persistent decode_kernel)
  int lwe_graph = 1;           // MLLM_LWE_GRAPH=0 launches the batched decode step without a CUDA graph
  int tmax = 0;                // token rows per forward (MLLM_LWE_TOKENS)
  LweArgs lw{};
  LweHost lh;
  Grow g_bids, g_plan, g_bout, g_state, g_blogits, g_spec;
  int32_t* h_active = nullptr; // pinned
  // cluster decode (cdec.cu): the single-token loop on one 16-CTA cluster per kv head, for the models
  // it supports
  int cd_ok = 0;
  int cd_nc = 1;               // clusters per launch (nKvHeads)
  CdSmem cd_plan{};            // the kernel's shared-memory plan
  size_t cd_smem = 0;
  uint8_t* d_cdw = nullptr;    // repacked weight chunks
  uint32_t* d_cdoff = nullptr; // [16 nc] first chunk of each CTA's stream
  uint32_t* d_cdcpt = nullptr; // [16 nc] chunks per token of each CTA
  uint32_t* d_cdcnt = nullptr; // [16 nc x 16] records per token of each warp
  uint64_t* d_cdgx = nullptr;  // exchange words between the clusters (nc > 1)
  size_t cd_gx_bytes = 0;
  uint32_t cd_launches = 0;    // launches since the exchange words were last zeroed
  mutable char kernel_desc[64] = {};
  // token streaming (mllm_generate_stream): ids published by the kernels into mapped pinned memory
  int32_t* h_stream = nullptr; // host view: [0] count, [kStreamHead + i] id i | phase << 30
  int32_t* d_stream = nullptr; // the same words, device view
  mllm_token_fn on_token = nullptr;
  void* on_token_user = nullptr;
  int delivered = 0;           // ids handed to on_token so far in this call
  long coop_launches = 0;      // persistent-kernel launches issued by this handle
  long spec_graph_kernels = 0; // kernels in one speculation graph replay
  long spec_captured = 0;      // kernels counted while capturing in this call (captured, not run)
  // the instantiated speculation step of the last call, kept while its arguments repeat
  cudaGraphExec_t spec_exec = nullptr;
  const void* spec_key_ptr[3] = {nullptr, nullptr, nullptr};  // sp, d_out, stream words
  int spec_key[5] = {0, 0, 0, 0, -1};                         // k, ngram, max_new, eos, slot
  long spec_replay_kernels = 0;
};

namespace {
// Kernel launches issued so far for handle e on this thread (persistent kernels + token-batch kernels).
long launches_now(const mllm_engine* e) { return e->coop_launches + lwe_launch_count(); }
}  // namespace

namespace {

int fail(mllm_engine* e, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (e) e->err = buf;
  else g_create_error = buf;
  return code;
}

#define CUDA_TRY(e, call)                                                                             \
  do {                                                                                                \
    cudaError_t _st = (call);                                                                         \
    if (_st != cudaSuccess) return fail(e, MLLM_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_st)); \
  } while (0)

template <class T>
int dev_alloc(mllm_engine* e, T** p, size_t bytes) {
  void* q = nullptr;
  bytes = std::max<size_t>(bytes, 16);
  cudaError_t st = cudaMalloc(&q, bytes);
  if (st != cudaSuccess) return fail(e, MLLM_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(st));
  e->allocs.push_back(q);
  e->bytes += bytes;
  *p = (T*)q;
  return MLLM_OK;
}

int grow(mllm_engine* e, Grow& g, size_t bytes) {
  bytes = std::max<size_t>(bytes, 256);
  if (g.cap >= bytes) return MLLM_OK;
  if (g.p) {
    CUDA_TRY(e, cudaStreamSynchronize(e->stream));
    cudaFree(g.p);
    e->bytes -= g.cap;
    g.p = nullptr;
    g.cap = 0;
  }
  cudaError_t st = cudaMalloc(&g.p, bytes);
  if (st != cudaSuccess) return fail(e, MLLM_ERR_OOM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(st));
  g.cap = bytes;
  e->bytes += bytes;
  return MLLM_OK;
}

#define TRY(x)                \
  do {                        \
    int _rc = (x);            \
    if (_rc != MLLM_OK) return _rc; \
  } while (0)

const PgwTensor* tensor(const PgwModel& m, const std::string& name) {
  auto it = m.tensors.find(name);
  return it == m.tensors.end() ? nullptr : &it->second;
}

int upload_q4(mllm_engine* e, const uint8_t* buf, const std::string& name, int rows, int cols, Q4* out) {
  const PgwTensor* t = tensor(e->pgw, name);
  if (!t) return fail(e, MLLM_ERR_FORMAT, "missing tensor %s", name.c_str());
  if (t->storage != "q4") return fail(e, MLLM_ERR_UNSUPPORTED, "%s is %s; this backend runs q4 only", name.c_str(), t->storage.c_str());
  if (t->shape.size() != 2 || t->shape[0] != rows || t->shape[1] != cols)
    return fail(e, MLLM_ERR_FORMAT, "%s has an unexpected shape", name.c_str());
  if (t->group != 32) return fail(e, MLLM_ERR_UNSUPPORTED, "%s uses group %d; only 32 is supported", name.c_str(), t->group);
  if (t->nbytes != (int64_t)rows * cols / 2 || t->scale_nbytes != (int64_t)rows * (cols / 32) * 4)
    return fail(e, MLLM_ERR_FORMAT, "%s: byte counts do not match its shape", name.c_str());
  uint32_t* w;
  float* s;
  TRY(dev_alloc(e, &w, t->nbytes));
  TRY(dev_alloc(e, &s, t->scale_nbytes));
  CUDA_TRY(e, cudaMemcpy(w, buf + e->pgw.payload_off + t->offset, t->nbytes, cudaMemcpyHostToDevice));
  CUDA_TRY(e, cudaMemcpy(s, buf + e->pgw.payload_off + t->scale_offset, t->scale_nbytes, cudaMemcpyHostToDevice));
  out->w = w;
  out->s = s;
  return MLLM_OK;
}

int upload_f32(mllm_engine* e, const uint8_t* buf, const std::string& name, int64_t count, const float** out,
               bool optional = false) {
  const PgwTensor* t = tensor(e->pgw, name);
  if (!t) {
    if (optional) {
      *out = nullptr;
      return MLLM_OK;
    }
    return fail(e, MLLM_ERR_FORMAT, "missing tensor %s", name.c_str());
  }
  if (t->storage != "f32") return fail(e, MLLM_ERR_UNSUPPORTED, "%s is %s, expected f32", name.c_str(), t->storage.c_str());
  if (t->nbytes < count * 4) return fail(e, MLLM_ERR_FORMAT, "%s is shorter than expected", name.c_str());
  float* d;
  TRY(dev_alloc(e, &d, count * 4));
  CUDA_TRY(e, cudaMemcpy(d, buf + e->pgw.payload_off + t->offset, count * 4, cudaMemcpyHostToDevice));
  *out = d;
  return MLLM_OK;
}

// engine/infer.js:185-206: f32 inverse frequencies, f64 cos/sin, f32 tables duplicated over halves.
void build_rope(int max_seq, int head_dim, double theta, double pct, std::vector<float>* cs, std::vector<float>* sn,
                int* rope_dim) {
  int rd = (int)std::floor(head_dim * pct);
  rd -= rd % 2;
  const int half = rd / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = (float)(1.0 / std::pow(theta, (double)(2 * i) / rd));
  cs->assign((size_t)max_seq * std::max(rd, 1), 0.f);
  sn->assign((size_t)max_seq * std::max(rd, 1), 0.f);
  for (int t = 0; t < max_seq; ++t)
    for (int i = 0; i < half; ++i) {
      const double f = (double)t * inv[i];
      const float c = (float)std::cos(f), s = (float)std::sin(f);
      (*cs)[(size_t)t * rd + i] = c;
      (*cs)[(size_t)t * rd + half + i] = c;
      (*sn)[(size_t)t * rd + i] = s;
      (*sn)[(size_t)t * rd + half + i] = s;
    }
  *rope_dim = rd;
}

int check_slot(mllm_engine* e, int slot) {
  if (slot < 0 || slot >= (int)e->slots.size()) return fail(e, MLLM_ERR_ARG, "slot %d out of range [0, %zu)", slot, e->slots.size());
  return MLLM_OK;
}

// Launch one of the two decode kernels.  `resume` continues an earlier launch on the same stream:
// its status words and error flag are kept (the earlier launch's error stops this one at entry).
int launch(mllm_engine* e, RunArgs& a, int max_forwards, bool multi, bool resume = false) {
  a.m = e->md;
  a.x = e->ex;
  a.mmax = e->mmax;
  a.srows = multi ? e->mmax : 1;
  a.status = e->d_status;
  a.err = e->d_err;
  // Tags only grow; when the 32-bit space would wrap, clear every exchange word and restart at 1.
  if ((uint64_t)e->tag + (uint64_t)max_forwards + 2 >= 0xFFFFFFF0ull) {
    CUDA_TRY(e, cudaStreamSynchronize(e->stream));
    const size_t L = e->md.n_layers, M = e->mmax;
    CUDA_TRY(e, cudaMemset(e->ex.qkv, 0, L * M * e->ex.s_qkv * 8));
    CUDA_TRY(e, cudaMemset(e->ex.att, 0, L * M * e->ex.s_d * 8));
    CUDA_TRY(e, cudaMemset(e->ex.x1, 0, L * M * e->ex.s_d * 8));
    CUDA_TRY(e, cudaMemset(e->ex.a, 0, L * M * e->ex.s_ff * 8));
    CUDA_TRY(e, cudaMemset(e->ex.x2, 0, L * M * e->ex.s_d * 8));
    CUDA_TRY(e, cudaMemset(e->ex.cand, 0, (attn_partials_offset(e->grid, (int)M) + attn_partials_words(L, e->md.NH)) * 8));
    e->tag = 1;
  }
  a.base_tag = e->tag;
  e->tag += (uint32_t)max_forwards + 2;
  a.poll_sleep_ns = e->poll_sleep_ns;
  a.weight_policy = e->weight_policy;
  a.l2_prefetch = e->l2_prefetch;
  a.lm_rpc = multi ? 0 : e->lm_rpc;
  if (!resume) {
    CUDA_TRY(e, cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream));
    CUDA_TRY(e, cudaMemsetAsync(e->d_status, 0, ST_WORDS * sizeof(int32_t), e->stream));
  }
  // the single-token kernel with position-split attention only when a position of the call can need
  // kAttnMinRounds rounds of the attention loop
  const int maxpos = a.mode == MODE_GENERATE ? a.n_ids + a.max_new : a.pos0 + 1;
  const bool split = maxpos > kAttnRound * (kAttnMinRounds - 1);
  if (!multi && e->cd_ok) {
    CdArgs ca;
    ca.r = a;
    ca.wst = e->d_cdw;
    ca.woff = e->d_cdoff;
    ca.wcpt = e->d_cdcpt;
    ca.wcnt = e->d_cdcnt;
    ca.L = e->cd_plan;
    ca.nc = e->cd_nc;
    ca.gx = e->d_cdgx;
    // each launch owns 2^22 tags of the exchange words; after 2^10 launches the words are zeroed
    // and the tags start over
    if (e->d_cdgx && e->cd_launches % 1024u == 0)
      CUDA_TRY(e, cudaMemsetAsync(e->d_cdgx, 0, e->cd_gx_bytes, e->stream));
    ca.tag0 = (e->cd_launches % 1024u) << 22;
    ++e->cd_launches;
    const cudaError_t lst = cd_launch(ca, e->cd_smem, e->stream);
    ++e->coop_launches;
    if (lst != cudaSuccess) return fail(e, MLLM_ERR_CUDA, "cluster decode launch failed: %s", cudaGetErrorString(lst));
    return MLLM_OK;
  }
  DecodeFn k = multi ? e->kernel_multi : split ? e->kernel_single_split : e->kernel_single;
  const size_t smem = multi ? e->smem_multi : e->smem_single;
  void* args[] = {&a};
  cudaError_t lst = cudaLaunchCooperativeKernel((void*)k, e->grid, kThreads, args, smem, e->stream);
  ++e->coop_launches;
  if (lst != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, (const void*)k);
    int per_sm = -1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem);
    return fail(e, MLLM_ERR_CUDA,
                "cooperative launch failed: %s (grid %d, smem %zu, regs %d, maxThreads %d, maxDynSmem %d, "
                "static smem %zu, local %zu, params %zu B, blocks/SM %d)",
                cudaGetErrorString(lst), e->grid, smem, fa.numRegs, fa.maxThreadsPerBlock,
                fa.maxDynamicSharedSizeBytes, fa.sharedSizeBytes, fa.localSizeBytes, sizeof(RunArgs), per_sm);
  }
  return MLLM_OK;
}

int fetch_status(mllm_engine* e) {
  CUDA_TRY(e, cudaMemcpyAsync(e->h_status, e->d_status, ST_WORDS * sizeof(int32_t), cudaMemcpyDeviceToHost, e->stream));
  CUDA_TRY(e, cudaMemcpyAsync(e->h_status + ST_WORDS, e->d_err, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  return MLLM_OK;
}

// Hand the ids published since the last call to the caller's on_token (streaming calls only).
void deliver(mllm_engine* e) {
  if (!e->on_token) return;
  const int n = *reinterpret_cast<volatile int32_t*>(e->h_stream);
  std::atomic_thread_fence(std::memory_order_acquire);
  for (; e->delivered < n; ++e->delivered) {
    const uint32_t v = (uint32_t) reinterpret_cast<volatile int32_t*>(e->h_stream)[kStreamHead + e->delivered];
    e->on_token((int32_t)(v & 0x3FFFFFFFu), e->delivered, (int32_t)(v >> 30), e->on_token_user);
  }
}

// Wait for the handle's stream; while it runs, ids published by the kernels go to on_token as they
// land (streaming calls) instead of after the launch.
cudaError_t wait_stream(mllm_engine* e) {
  if (!e->on_token) return cudaStreamSynchronize(e->stream);
  for (;;) {
    deliver(e);
    const cudaError_t q = cudaStreamQuery(e->stream);
    if (q != cudaErrorNotReady) {
      deliver(e);
      return q;
    }
    std::this_thread::yield();
  }
}

int finish(mllm_engine* e) {
  CUDA_TRY(e, wait_stream(e));
  if (e->h_status[ST_WORDS] != 0) {
    // a CTA that gave up may have left a completion counter of the token-batch kernels non-zero
    cudaMemset(e->lh.attn_ctr, 0, e->lh.attn_ctr_n * sizeof(int));
    cudaMemset(e->lw.skctr, 0, kLweSplitKTiles * sizeof(int));
  }
  if (e->h_status[ST_WORDS] == 2) return fail(e, MLLM_ERR_ARG, "a prompt token id is out of range");
  if (e->h_status[ST_WORDS] == kCdShapeError)
    return fail(e, MLLM_ERR_CUDA, "cluster decode ran with a launch shape other than its clusters of %d CTAs", kCdCtas);
  if (e->h_status[ST_WORDS] != 0)
    return fail(e, MLLM_ERR_TIMEOUT, "a device-side wait exceeded its time limit; the call was abandoned");
  return MLLM_OK;
}

uint64_t u64_at(const int32_t* s, int i) { return (uint64_t)(uint32_t)s[i] | ((uint64_t)(uint32_t)s[i + 1] << 32); }

LweArgs lwe_args(const mllm_engine* e) {
  LweArgs a = e->lw;
  a.m = e->md;
  a.err = e->d_err;
  return a;
}

// Token-batch forward of n device ids of one slot at positions pos0.. in chunks of tmax tokens
// (engine/infer.js:553-577 for every token).  The lm_head runs on the last token (argmax -> d_amax[0],
// logits [V]) or, with lm_each, on every token (d_amax[i], logits [n][V]).  Returns the forward count.
int lwe_run(mllm_engine* e, int slot, const int32_t* d_ids, int n, int pos0, int lm_each, float* d_logits,
            int32_t* d_amax, int* forwards) {
  const Slot& s = e->slots[slot];
  (void)s;
  LweArgs a = lwe_args(e);
  const int V = e->md.vocab;
  int f = 0;
  for (int c0 = 0; c0 < n; c0 += e->tmax) {
    const int Tc = std::min(e->tmax, n - c0);
    const bool last = c0 + Tc >= n;
    lwe_fill(a, d_ids + c0, Tc, slot, pos0 + c0, lm_each, e->stream);
    LweArgs b = a;
    b.amax = d_amax + (lm_each ? c0 : 0);
    const int lm_T = lm_each ? Tc : (last ? 1 : 0);
    float* lg = d_logits && lm_T ? d_logits + (size_t)(lm_each ? c0 : 0) * V : nullptr;
    CUDA_TRY(e, lwe_forward(b, e->lh, Tc, lm_T, !lm_each, lg, false, e->stream));
    ++f;
  }
  *forwards = f;
  return MLLM_OK;
}

// Prompt-lookup speculation after a token-batch prefill (first id already in d_out[0]): iterations of
// draft lookup -> (k + 1)-row verify forward -> accept, one CUDA graph replay each, state on the
// device; the host only checks the done word every few replays.
int spec_loop(mllm_engine* e, int slot, const int32_t* d_ids, int n, int max_new, int32_t eos, int k, int ngram,
              int32_t* d_out, int prefill_forwards) {
  cudaStream_t st = e->stream;
  TRY(grow(e, e->g_spec, (size_t)(kSpecHist + e->md.kv_len + 128) * 4));
  int32_t* sp = (int32_t*)e->g_spec.p;
  lwe_spec_init(sp, d_ids, n, d_out, max_new, eos, e->md.kv_len, prefill_forwards, st);
  const LweArgs a = lwe_args(e);
  int32_t* sid = e->on_token ? e->d_stream : nullptr;
  cudaGraphExec_t exec = nullptr;
  if (e->lwe_graph) {
    // The step's kernels and their arguments depend only on these values (the engine's buffers are
    // fixed), so a repeated call replays the graph instantiated by the previous one.
    const void* kp[3] = {sp, d_out, sid};
    const int kv[5] = {k, ngram, max_new, eos, slot};
    if (!e->spec_exec || memcmp(kp, e->spec_key_ptr, sizeof kp) || memcmp(kv, e->spec_key, sizeof kv)) {
      if (e->spec_exec) cudaGraphExecDestroy(e->spec_exec);
      e->spec_exec = nullptr;
      cudaGraph_t graph = nullptr;
      CUDA_TRY(e, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      const long c0 = launches_now(e);
      const cudaError_t r1 = lwe_spec_iteration(a, e->lh, sp, d_out, k, ngram, max_new, eos, slot, sid, st);
      e->spec_graph_kernels = e->spec_captured = launches_now(e) - c0;
      const cudaError_t r2 = cudaStreamEndCapture(st, &graph);
      if (r1 != cudaSuccess || r2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return fail(e, MLLM_ERR_CUDA, "capture of the speculation step failed: %s",
                    cudaGetErrorString(r1 != cudaSuccess ? r1 : r2));
      }
      const cudaError_t r3 = cudaGraphInstantiate(&e->spec_exec, graph, 0);
      cudaGraphDestroy(graph);
      if (r3 != cudaSuccess) {
        e->spec_exec = nullptr;
        return fail(e, MLLM_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(r3));
      }
      memcpy(e->spec_key_ptr, kp, sizeof kp);
      memcpy(e->spec_key, kv, sizeof kv);
    }
    exec = e->spec_exec;
  }
  cudaError_t rs = cudaSuccess;
  long replays = 0;
  for (int it = (int)replays; it < max_new + 1 && rs == cudaSuccess;) {
    for (int b = 0; b < 4 && rs == cudaSuccess; ++b, ++it, ++replays)
      rs = exec ? cudaGraphLaunch(exec, st) : lwe_spec_iteration(a, e->lh, sp, d_out, k, ngram, max_new, eos, slot, sid, st);
    if (rs == cudaSuccess) rs = cudaMemcpyAsync(e->h_active, sp + kSpecDoneWord, 4, cudaMemcpyDeviceToHost, st);
    if (rs == cudaSuccess) rs = wait_stream(e);
    if (rs == cudaSuccess && *e->h_active) break;
  }
  if (exec) e->spec_replay_kernels = replays * e->spec_graph_kernels;
  if (rs != cudaSuccess) return fail(e, MLLM_ERR_CUDA, "speculation step: %s", cudaGetErrorString(rs));
  lwe_spec_finish(sp, e->d_status, st);
  return MLLM_OK;
}

int generate_impl(mllm_engine* e, int slot, const int32_t* d_ids, int n, int max_new, int32_t eos, int spec_k,
                  int ngram, int32_t* d_out, mllm_stats* st) {
  TRY(check_slot(e, slot));
  const long l0 = launches_now(e);
  if (n <= 0 || max_new <= 0) return fail(e, MLLM_ERR_ARG, "empty prompt or max_new <= 0");
  if (n > e->md.kv_len - 1)
    return fail(e, MLLM_ERR_ARG, "prompt of %d ids does not fit the %d-position cache", n, e->md.kv_len);
  if (spec_k < 0 || (spec_k > 0 && ngram <= 0)) return fail(e, MLLM_ERR_ARG, "bad speculation settings");
  if (spec_k > 0 && e->md.arch == 1)
    return fail(e, MLLM_ERR_UNSUPPORTED, "prompt-lookup speculation runs on llama-arch files only");
  Slot& s = e->slots[slot];
  RunArgs a{};
  a.kc = s.k;
  a.vc = s.v;
  a.mode = MODE_GENERATE;
  a.ids = d_ids;
  a.n_ids = n;
  a.max_new = max_new;
  a.eos = eos;
  a.spec_k = spec_k;
  a.ngram = ngram;
  a.out_ids = d_out;
  a.stream_ids = e->on_token ? e->d_stream : nullptr;
  const int chunks = (n + e->mmax - 1) / e->mmax;
  if (e->lwe_ok) {
    // Prefill as token-batch forwards on the tensor cores, first id from its argmax, then the decode
    // loop (greedy: the single-token kernel; speculative: the general kernel) resumes from out_ids.
    CUDA_TRY(e, cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream));
    CUDA_TRY(e, cudaMemsetAsync(e->d_status, 0, ST_WORDS * sizeof(int32_t), e->stream));
    lwe_mark_time(e->d_status, ST_T0, e->stream);
    int f = 0;
    TRY(lwe_run(e, slot, d_ids, n, 0, 0, nullptr, e->lw.amax, &f));
    lwe_first(lwe_args(e), d_out, e->d_status, eos, f, a.stream_ids, e->stream);
    if (spec_k > 0) {
      e->spec_captured = e->spec_replay_kernels = 0;
      TRY(spec_loop(e, slot, d_ids, n, max_new, eos, std::min(spec_k, kSpecMaxK), ngram, d_out, f));
    } else if (max_new > 1) {
      a.start_gen = 1;
      TRY(launch(e, a, max_new + 1, false, true));
    }
  } else if (spec_k > 0) {
    TRY(launch(e, a, chunks + max_new + 1, true));
  } else {
    // Prefill on the general kernel, then the greedy loop on the single-token kernel; the second
    // launch follows on the same stream and picks up the first id from out_ids.
    a.prefill_only = 1;
    TRY(launch(e, a, chunks, true));
    if (max_new > 1) {
      RunArgs b = a;
      b.prefill_only = 0;
      b.start_gen = 1;
      TRY(launch(e, b, max_new, false, true));
    }
  }
  TRY(fetch_status(e));
  TRY(finish(e));
  const int32_t* hs = e->h_status;
  const int gen = hs[ST_NGEN];
  // engine/webgpu.js:1215-1218 style cache bookkeeping: every accepted id has its K/V in the cache
  // except the last one generated.
  s.cache_len = std::min(n + gen - 1, e->md.kv_len);
  if (st) {
    st->n_generated = gen;
    st->stop_reason = hs[ST_STOP];
    st->spec_hits = hs[ST_HITS];
    st->spec_tries = hs[ST_TRIES];
    st->forwards = hs[ST_FORWARDS];
    st->prompt_len = n;
    const uint64_t t0 = u64_at(hs, ST_T0), t1 = u64_at(hs, ST_TFIRST), t2 = u64_at(hs, ST_TEND);
    st->ttft_ms = t1 > t0 ? (float)((t1 - t0) * 1e-6) : 0.f;
    st->total_ms = t2 > t0 ? (float)((t2 - t0) * 1e-6) : 0.f;
    // graph replays ran spec_graph_kernels kernels each; the capture itself ran none
    st->kernel_launches =
        (int32_t)(launches_now(e) - l0 - (spec_k > 0 ? e->spec_captured - e->spec_replay_kernels : 0));
  }
  return MLLM_OK;
}

}  // namespace

extern "C" {

const char* mllm_last_error(const mllm_engine* e) { return e ? e->err.c_str() : g_create_error.c_str(); }

void mllm_destroy(mllm_engine* e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (void* p : e->allocs) cudaFree(p);
  for (Grow* g : {&e->g_bids, &e->g_plan, &e->g_bout, &e->g_state, &e->g_blogits, &e->g_spec})
    if (g->p) cudaFree(g->p);
  if (e->h_status) cudaFreeHost(e->h_status);
  if (e->h_active) cudaFreeHost(e->h_active);
  if (e->h_stream) cudaFreeHost(e->h_stream);
  if (e->spec_exec) cudaGraphExecDestroy(e->spec_exec);
  if (e->own_stream) cudaStreamDestroy(e->own_stream);
  delete e;
}

int mllm_create(int device, const uint8_t* buf, size_t len, int max_slots, int kv_len, mllm_engine** out) {
  if (!out) return fail(nullptr, MLLM_ERR_ARG, "out is null");
  *out = nullptr;
  std::unique_ptr<mllm_engine, void (*)(mllm_engine*)> e(new mllm_engine(), mllm_destroy);
  std::string perr;
  if (!parse_pgw(buf, len, &e->pgw, &perr)) return fail(nullptr, MLLM_ERR_FORMAT, "%s", perr.c_str());
  PgwModel& p = e->pgw;
  auto bad = [&](int code, const char* msg) { return fail(nullptr, code, "%s", msg); };
  if (p.kind != "q4") return bad(MLLM_ERR_UNSUPPORTED, "only q4 PGW files are supported by this backend");
  if (p.n_layers <= 0 || p.d_model <= 0 || p.n_heads <= 0 || p.n_kv_heads <= 0 || p.vocab <= 0 || p.max_seq <= 1)
    return bad(MLLM_ERR_FORMAT, "header holds a zero dimension");
  if (p.d_model % p.n_heads || p.d_model / p.n_heads != kHeadDim)
    return bad(MLLM_ERR_UNSUPPORTED, "head_dim must be 64");
  if (p.n_heads % p.n_kv_heads) return bad(MLLM_ERR_FORMAT, "nHeads is not a multiple of nKvHeads");
  if (p.d_model % 32 || p.d_ff % 32) return bad(MLLM_ERR_UNSUPPORTED, "dModel and dFf must be multiples of 32");
  if (max_slots <= 0) return bad(MLLM_ERR_ARG, "max_slots must be positive");
  e->device = device;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return bad(MLLM_ERR_CUDA, "no CUDA device available");
  if (device < 0 || device >= ndev) return bad(MLLM_ERR_ARG, "device index out of range");
  if (cudaSetDevice(device) != cudaSuccess) return bad(MLLM_ERR_CUDA, "cudaSetDevice failed");
  ModelDev& md = e->md;
  md.arch = p.arch;
  md.vocab = p.vocab;
  md.n_layers = p.n_layers;
  md.D = p.d_model;
  md.NH = p.n_heads;
  md.NKV = p.n_kv_heads;
  md.FF = p.d_ff;
  md.QKV = md.D + 2 * md.NKV * kHeadDim;
  md.max_seq = p.max_seq;
  md.kv_len = kv_len > 0 ? std::min(kv_len, p.max_seq) : p.max_seq;
  e->kernel_multi = pick_decode_kernel(md.D, md.FF, true);
  e->kernel_single = pick_decode1_kernel(md.D, md.FF, false);
  e->kernel_single_split = pick_decode1_kernel(md.D, md.FF, true);
  if (!e->kernel_multi || !e->kernel_single || !e->kernel_single_split) return bad(MLLM_ERR_UNSUPPORTED, "dModel/dFf beyond the kernel limits (1024 / 4096)");
  mllm_engine* E = e.get();
  auto relay = [&](int rc) {
    if (rc != MLLM_OK) g_create_error = E->err;
    return rc;
  };
  // ---- weights
  const int D = md.D, FF = md.FF, L = md.n_layers;
  std::vector<LayerDev> layers(L);
  for (int l = 0; l < L; ++l) {
    const std::string b = "blocks." + std::to_string(l) + ".";
    LayerDev& ld = layers[l];
    int rc;
    if ((rc = upload_q4(E, buf, b + "attn.qkv", md.QKV, D, &ld.qkv))) return relay(rc);
    if ((rc = upload_q4(E, buf, b + "attn.proj", D, D, &ld.proj))) return relay(rc);
    if (md.arch == 0) {
      if ((rc = upload_q4(E, buf, b + "mlp.w1", FF, D, &ld.w1))) return relay(rc);
      if ((rc = upload_q4(E, buf, b + "mlp.w3", FF, D, &ld.w3))) return relay(rc);
      if ((rc = upload_q4(E, buf, b + "mlp.w2", D, FF, &ld.w2))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "norm1", D, &ld.norm1))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "norm2", D, &ld.norm2))) return relay(rc);
    } else {
      if ((rc = upload_q4(E, buf, b + "mlp.fc", FF, D, &ld.w1))) return relay(rc);
      if ((rc = upload_q4(E, buf, b + "mlp.proj", D, FF, &ld.w2))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "ln1", 2 * D, &ld.norm1))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "ln2", 2 * D, &ld.norm2))) return relay(rc);
      // engine/infer.js:173-176: a missing bias is skipped
      if ((rc = upload_f32(E, buf, b + "attn.qkv_bias", md.QKV, &ld.qkv_b, true))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "attn.proj_bias", D, &ld.proj_b, true))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "mlp.fc_bias", FF, &ld.fc_b, true))) return relay(rc);
      if ((rc = upload_f32(E, buf, b + "mlp.proj_bias", D, &ld.mproj_b, true))) return relay(rc);
    }
  }
  {
    int rc;
    if ((rc = upload_q4(E, buf, "lm_head", md.vocab, D, &md.lm))) return relay(rc);
    if (md.arch == 0) {
      if ((rc = upload_f32(E, buf, "norm_f", D, &md.norm_f))) return relay(rc);
    } else {
      if ((rc = upload_f32(E, buf, "ln_f", 2 * D, &md.norm_f))) return relay(rc);
      if ((rc = upload_f32(E, buf, "wpe", (int64_t)md.max_seq * D, &md.wpe))) return relay(rc);
      if ((rc = upload_f32(E, buf, "scale_factors", D, &md.sf, true))) return relay(rc);
    }
    LayerDev* dl;
    if ((rc = dev_alloc(E, &dl, sizeof(LayerDev) * L))) return relay(rc);
    if (cudaMemcpy(dl, layers.data(), sizeof(LayerDev) * L, cudaMemcpyHostToDevice) != cudaSuccess)
      return bad(MLLM_ERR_CUDA, "upload of layer table failed");
    md.layers = dl;
    if (md.arch == 0) {
      std::vector<float> cs, sn;
      build_rope(md.max_seq, kHeadDim, p.rope_theta, p.rope_pct, &cs, &sn, &md.rope_dim);
      float *dc, *ds;
      if ((rc = dev_alloc(E, &dc, cs.size() * 4)) || (rc = dev_alloc(E, &ds, sn.size() * 4))) return relay(rc);
      cudaMemcpy(dc, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(ds, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
      md.rope_cos = dc;
      md.rope_sin = ds;
    }
  }
  // ---- launch geometry: one CTA per SM, co-resident (cooperative launch)
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return bad(MLLM_ERR_CUDA, "cudaGetDeviceProperties failed");
  if (!prop.cooperativeLaunch) return bad(MLLM_ERR_CUDA, "device lacks cooperative launch");
  e->grid = prop.multiProcessorCount;
  const size_t smem_cap = prop.sharedMemPerBlockOptin;
  int mmax = 16;
  while (mmax > 1 && decode_smem_bytes(md, mmax, e->grid) > smem_cap) --mmax;
  e->mmax = mmax;
  e->smem_multi = decode_smem_bytes(md, mmax, e->grid);
  // lm_head rows resident in the single-token kernel's shared memory when they fit (MLLM_LM_RESIDENT=0: off)
  {
    const int rpc = (md.vocab + e->grid - 1) / e->grid;
    bool want = true;
    if (const char* v = getenv("MLLM_LM_RESIDENT")) want = atoi(v) != 0;
    e->lm_rpc = want && decode1_smem_bytes(md, e->grid, rpc) <= smem_cap ? rpc : 0;
  }
  e->smem_single = decode1_smem_bytes(md, e->grid, e->lm_rpc);
  if (e->smem_multi > smem_cap) return bad(MLLM_ERR_UNSUPPORTED, "model does not fit the shared-memory budget");
  for (DecodeFn k : {e->kernel_multi, e->kernel_single, e->kernel_single_split}) {
    // The limit is an attribute of the kernel function, shared by every engine that uses the same
    // instantiation, so it is set to the device maximum rather than to this engine's need.
    if (cudaFuncSetAttribute((const void*)k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_cap) != cudaSuccess)
      return bad(MLLM_ERR_CUDA, "cudaFuncSetAttribute failed");
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, k == e->kernel_multi ? e->smem_multi : e->smem_single);
    if (per_sm < 1) return bad(MLLM_ERR_CUDA, "decode kernel cannot be resident with its shared memory");
  }
  // ---- cluster decode: weights repacked into per-(CTA, warp) streams (MLLM_CLUSTER_DECODE=1: on, with
  // as many clusters as the device holds at once; =N with N > 1: at most max(N, nKvHeads) clusters)
  {
    int cap = 0;
    if (const char* v = getenv("MLLM_CLUSTER_DECODE")) cap = atoi(v);
    const bool want = cap != 0;
    cap = cap > 1 ? std::max(cap, md.NKV) : kCdMaxClusters;
    int nc = 0;
    if (want && cd_setup(smem_cap) == cudaSuccess)
      for (nc = std::min(cap, kCdMaxClusters); nc >= md.NKV && nc >= 1; --nc)
        if (cd_supported(md, smem_cap, nc) && cd_max_clusters(cd_smem_bytes(md, smem_cap, nc)) >= nc) break;
    if (want && nc >= md.NKV && nc >= 1) {
      auto host_q4 = [&](const std::string& name, int rows, int cols) {
        const PgwTensor* t = tensor(p, name);
        return HostQ4{buf + p.payload_off + t->offset, buf + p.payload_off + t->scale_offset, rows, cols};
      };
      std::vector<HostQ4> mats;
      for (int l = 0; l < L; ++l) {
        const std::string b = "blocks." + std::to_string(l) + ".";
        mats.push_back(host_q4(b + "attn.qkv", md.QKV, D));
        mats.push_back(host_q4(b + "attn.proj", D, D));
        mats.push_back(host_q4(b + "mlp.w1", FF, D));
        mats.push_back(host_q4(b + "mlp.w3", FF, D));
        mats.push_back(host_q4(b + "mlp.w2", D, FF));
      }
      std::vector<uint8_t> packed;
      std::vector<uint32_t> off, cpt, cnt;
      cd_pack(md, nc, mats, host_q4("lm_head", md.vocab, D), &packed, &off, &cpt, &cnt);
      int rc;
      if ((rc = dev_alloc(E, &e->d_cdw, packed.size())) || (rc = dev_alloc(E, &e->d_cdoff, off.size() * 4)) ||
          (rc = dev_alloc(E, &e->d_cdcpt, cpt.size() * 4)) || (rc = dev_alloc(E, &e->d_cdcnt, cnt.size() * 4)))
        return relay(rc);
      if (nc > 1) {
        e->cd_gx_bytes = cd_gx_words(md, nc, -1) * 8;
        if ((rc = dev_alloc(E, &e->d_cdgx, e->cd_gx_bytes))) return relay(rc);
      }
      cudaMemcpy(e->d_cdw, packed.data(), packed.size(), cudaMemcpyHostToDevice);
      cudaMemcpy(e->d_cdoff, off.data(), off.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(e->d_cdcpt, cpt.data(), cpt.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(e->d_cdcnt, cnt.data(), cnt.size() * 4, cudaMemcpyHostToDevice);
      e->cd_smem = cd_smem_bytes(md, smem_cap, nc);
      e->cd_plan = cd_smem(md, (int)smem_cap, nc);
      e->cd_nc = nc;
      e->cd_ok = 1;
    }
  }
  // ---- exchange buffers
  {
    auto pad = [](int n) { return (n + 31) & ~31; };
    ExchangeDev& x = e->ex;
    x.s_qkv = pad(md.QKV);
    x.s_d = pad(D);
    x.s_ff = pad(FF);
    const size_t LM = (size_t)L * mmax;
    int rc;
    if ((rc = dev_alloc(E, &x.qkv, LM * x.s_qkv * 8)) || (rc = dev_alloc(E, &x.att, LM * x.s_d * 8)) ||
        (rc = dev_alloc(E, &x.x1, LM * x.s_d * 8)) || (rc = dev_alloc(E, &x.a, LM * x.s_ff * 8)) ||
        (rc = dev_alloc(E, &x.x2, LM * x.s_d * 8)) || (rc = dev_alloc(E, &x.cand, (attn_partials_offset(e->grid, mmax) + attn_partials_words(L, md.NH)) * 8)))
      return relay(rc);
    cudaMemset(x.qkv, 0, LM * x.s_qkv * 8);
    cudaMemset(x.att, 0, LM * x.s_d * 8);
    cudaMemset(x.x1, 0, LM * x.s_d * 8);
    cudaMemset(x.a, 0, LM * x.s_ff * 8);
    cudaMemset(x.x2, 0, LM * x.s_d * 8);
    cudaMemset(x.cand, 0, (attn_partials_offset(e->grid, mmax) + attn_partials_words(L, md.NH)) * 8);
  }
  // ---- per-slot KV caches (engine/infer.js:348-358 layout per layer: [nKv][maxSeq][hd])
  e->slots.resize(max_slots);
  const size_t kvn = (size_t)L * md.NKV * md.kv_len * kHeadDim;
  for (auto& s : e->slots) {
    int rc;
    if ((rc = dev_alloc(E, &s.k, kvn * 4)) || (rc = dev_alloc(E, &s.v, kvn * 4))) return relay(rc);
    cudaMemset(s.k, 0, kvn * 4);
    cudaMemset(s.v, 0, kvn * 4);
  }
  int rc;
  if ((rc = dev_alloc(E, &e->d_ids, (size_t)(md.kv_len + 16) * 4)) || (rc = dev_alloc(E, &e->d_out, (size_t)(md.kv_len + 16) * 4)) ||
      (rc = dev_alloc(E, &e->d_status, ST_WORDS * 4)) || (rc = dev_alloc(E, &e->d_err, 16)) ||
      (rc = dev_alloc(E, &e->d_argmax, (size_t)(md.kv_len + 16) * 4)))
    return relay(rc);
  if (cudaMallocHost(&e->h_status, (ST_WORDS + 1) * 4) != cudaSuccess) return bad(MLLM_ERR_OOM, "cudaMallocHost failed");
  if (cudaMallocHost(&e->h_active, 16) != cudaSuccess) return bad(MLLM_ERR_OOM, "cudaMallocHost failed");
  if (cudaHostAlloc(&e->h_stream, (size_t)(kStreamHead + md.kv_len + 32) * 4, cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(&e->d_stream, e->h_stream, 0) != cudaSuccess)
    return bad(MLLM_ERR_OOM, "mapped host buffer for token streaming failed");
  // ---- layer-wise engine buffers: tmax token rows per forward
  e->lwe_ok = md.NH / md.NKV <= kLweMaxRep;
  if (const char* v = getenv("MLLM_LWE_GRAPH")) e->lwe_graph = atoi(v) ? 1 : 0;
  if (const char* v = getenv("MLLM_LWE_FOLD_NORM")) e->lh.fold_norm = atoi(v) ? 1 : 0;
  if (const char* v = getenv("MLLM_LWE_ATTN_SPLIT")) e->lh.attn_split = atoi(v) ? 1 : 0;
  if (const char* v = getenv("MLLM_LWE_PDL")) e->lh.pdl = atoi(v);
  if (const char* v = getenv("MLLM_LWE_LM_WIDE")) e->lh.lm_wide = atoi(v);
  if (const char* v = getenv("MLLM_LWE_LM_TC5")) e->lh.lm_tc5 = atoi(v);
  if (const char* v = getenv("MLLM_LWE_GEMM_TC5")) e->lh.gemm_tc5 = atoi(v);
  if (const char* v = getenv("MLLM_LWE_ROPE_EPI")) e->lh.rope_epi = atoi(v);
  if (const char* v = getenv("MLLM_LWE_W13_WIDE")) e->lh.w13_wide = atoi(v);
  e->tmax = 1024;
  if (const char* v = getenv("MLLM_LWE_TOKENS")) e->tmax = std::max(16, std::min(8192, atoi(v)));
  e->lh.layers = layers;
  if (lwe_setup(md.kv_len) != cudaSuccess) return bad(MLLM_ERR_CUDA, "cudaFuncSetAttribute failed (token-batch kernels)");
  {
    LweArgs& w = e->lw;
    const size_t T = (e->tmax + 7) & ~7;  // whole 8-token blocks: the tiled halves of the tcgen05 lm_head
    auto r64 = [](int n) { return (n + 63) & ~63; };
    w.ldx = r64(std::max(D, md.NH * kHeadDim));
    w.ldx2 = r64(FF);
    w.lm_cap = e->tmax;
    const size_t nblk = (md.vocab + 63) / 64;
    float** kc;
    float** vc;
    int chunk, splits;
    lwe_attn_split_shape(md.kv_len, &chunk, &splits);
    const size_t rep = md.NH / md.NKV;
    // the position-split attention runs on decode steps (one row per slot) and short verify forwards
    const size_t arows = std::min<size_t>(T, std::max<size_t>(e->slots.size(), kLweSplitAttnRows));
    if ((rc = dev_alloc(E, &e->lh.attn_part, arows * md.NKV * splits * rep * 66 * 4)) ||
        (rc = dev_alloc(E, &e->lh.attn_ctr, arows * md.NKV * sizeof(int))))
      return relay(rc);
    e->lh.attn_ctr_n = arows * md.NKV;
    cudaMemset(e->lh.attn_ctr, 0, arows * md.NKV * sizeof(int));
    if ((rc = dev_alloc(E, &w.x, T * D * 4)) || (rc = dev_alloc(E, &w.xh, T * w.ldx * 2)) ||
        (rc = dev_alloc(E, &w.xl, T * w.ldx * 2)) || (rc = dev_alloc(E, &w.xh2, T * w.ldx2 * 2)) ||
        (rc = dev_alloc(E, &w.xl2, T * w.ldx2 * 2)) || (rc = dev_alloc(E, &w.qkv, T * md.QKV * 4)) ||
        (rc = dev_alloc(E, &w.xh3, T * w.ldx * 2)) || (rc = dev_alloc(E, &w.xl3, T * w.ldx * 2)) ||
        (rc = dev_alloc(E, &w.ss, T * kLweSsStride * 4)) || (rc = dev_alloc(E, &w.skws, kLweSkwsBytes)) ||
        (rc = dev_alloc(E, &w.skctr, kLweSplitKTiles * sizeof(int))) ||
        (rc = dev_alloc(E, &w.tok, T * 4)) || (rc = dev_alloc(E, &w.slot, T * 4)) || (rc = dev_alloc(E, &w.pos, T * 4)) ||
        (rc = dev_alloc(E, &w.lm_src, T * 4)) || (rc = dev_alloc(E, &w.amax, T * 4)) ||
        (rc = dev_alloc(E, &w.pval, nblk * T * 4)) || (rc = dev_alloc(E, &w.pidx, nblk * T * 4)) ||
        (rc = dev_alloc(E, &kc, e->slots.size() * sizeof(float*))) ||
        (rc = dev_alloc(E, &vc, e->slots.size() * sizeof(float*))))
      return relay(rc);
    cudaMemset(w.skctr, 0, kLweSplitKTiles * sizeof(int));
    std::vector<float*> hk, hv;
    for (auto& sl : e->slots) {
      hk.push_back(sl.k);
      hv.push_back(sl.v);
    }
    cudaMemcpy(kc, hk.data(), hk.size() * sizeof(float*), cudaMemcpyHostToDevice);
    cudaMemcpy(vc, hv.data(), hv.size() * sizeof(float*), cudaMemcpyHostToDevice);
    w.kc = kc;
    w.vc = vc;
  }
  if (e->lh.gemm_tc5 && md.arch == 0 && e->lwe_ok) {
    // the layer matrices expanded once into the tcgen05 tile's group images (fp16 hi/lo, swizzled)
    e->lh.pre.resize((size_t)L * kPreMats);
    for (int l = 0; l < L; ++l) {
      const LayerDev& Ld = layers[l];
      const Q4* mw[kPreMats] = {&Ld.qkv, &Ld.proj, &Ld.w1, &Ld.w2};
      const Q4* m3[kPreMats] = {nullptr, nullptr, &Ld.w3, nullptr};
      const int mr[kPreMats] = {md.QKV, D, FF, D}, mk[kPreMats] = {D, D, D, FF};
      for (int m = 0; m < kPreMats; ++m) {
        Tc5Pre& p = e->lh.pre[(size_t)l * kPreMats + m];
        const bool paired = m3[m] != nullptr;
        if ((rc = dev_alloc(E, &p.img, tc5_pre_bytes(mr[m], mk[m], paired))) ||
            (rc = dev_alloc(E, &p.down, (size_t)tc5_pre_tiles(mr[m], paired) * 4)))
          return relay(rc);
        if (tc5_expand(*mw[m], m3[m], mr[m], mk[m], p, 0) != cudaSuccess)
          return bad(MLLM_ERR_CUDA, "weight expansion for the tcgen05 GEMMs failed");
      }
    }
  }
  if (const char* v = getenv("MLLM_POLL_SLEEP_NS")) e->poll_sleep_ns = atoi(v);
  if (const char* v = getenv("MLLM_WEIGHT_EVICT_LAST")) e->weight_policy = atoi(v) ? 1 : 0;
  if (const char* v = getenv("MLLM_L2_PREFETCH")) e->l2_prefetch = atoi(v) ? 1 : 0;
  if (cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking) != cudaSuccess) return bad(MLLM_ERR_CUDA, "stream creation failed");
  e->stream = e->own_stream;
  if (cudaDeviceSynchronize() != cudaSuccess) return bad(MLLM_ERR_CUDA, "device error during upload");
  *out = e.release();
  return MLLM_OK;
}

int mllm_config(const mllm_engine* e, int32_t* c) {
  if (!e || !c) return MLLM_ERR_ARG;
  const ModelDev& m = e->md;
  const int32_t v[10] = {m.arch, m.vocab, m.n_layers, m.D, m.NH, m.NKV, m.FF, m.max_seq, m.kv_len, e->mmax};
  memcpy(c, v, sizeof v);
  return MLLM_OK;
}

size_t mllm_bytes_allocated(const mllm_engine* e) { return e ? e->bytes : 0; }

const char* mllm_decode_kernel(const mllm_engine* e) {
  if (!e) return "";
  if (e->cd_ok)
    snprintf(e->kernel_desc, sizeof(e->kernel_desc), "cdec_kernel: %d cluster(s) of %d CTAs", e->cd_nc, kCdCtas);
  else
    snprintf(e->kernel_desc, sizeof(e->kernel_desc), "decode1: grid of %d CTAs", e->grid);
  return e->kernel_desc;
}

int mllm_set_stream(mllm_engine* e, void* stream) {
  if (!e) return MLLM_ERR_ARG;
  cudaSetDevice(e->device);
  CUDA_TRY(e, cudaStreamSynchronize(e->stream));
  e->stream = stream ? (cudaStream_t)stream : e->own_stream;
  return MLLM_OK;
}

int mllm_reset(mllm_engine* e, int slot) {
  if (!e) return MLLM_ERR_ARG;
  TRY(check_slot(e, slot));
  e->slots[slot].cache_len = 0;
  return MLLM_OK;
}

int mllm_cache_len(const mllm_engine* e, int slot) {
  if (!e || slot < 0 || slot >= (int)e->slots.size()) return MLLM_ERR_ARG;
  return e->slots[slot].cache_len;
}

int mllm_forward(mllm_engine* e, int slot, const int32_t* ids, int n, int pos0, int logits_each, float* logits,
                 int32_t* argmax) {
  if (!e) return MLLM_ERR_ARG;
  cudaSetDevice(e->device);
  TRY(check_slot(e, slot));
  if (!ids || n <= 0) return fail(e, MLLM_ERR_ARG, "empty token list");
  if (pos0 < 0 || pos0 + n > e->md.kv_len)
    return fail(e, MLLM_ERR_ARG, "positions %d..%d exceed the %d-position cache", pos0, pos0 + n - 1, e->md.kv_len);
  if (pos0 > e->slots[slot].cache_len)
    return fail(e, MLLM_ERR_ARG, "pos0 %d leaves a gap after cacheLen %d", pos0, e->slots[slot].cache_len);
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= e->md.vocab) return fail(e, MLLM_ERR_ARG, "token id %d out of range", ids[i]);
  const size_t need = (size_t)(logits_each ? n : 1) * e->md.vocab;
  if (logits && need > e->logits_cap) {
    float* p;
    TRY(dev_alloc(e, &p, need * 4));
    e->d_logits = p;
    e->logits_cap = need;
  }
  CUDA_TRY(e, cudaMemcpyAsync(e->d_ids, ids, n * 4, cudaMemcpyHostToDevice, e->stream));
  Slot& s = e->slots[slot];
  RunArgs a{};
  a.kc = s.k;
  a.vc = s.v;
  a.mode = MODE_FORWARD;
  a.ids = e->d_ids;
  a.n_ids = n;
  a.pos0 = pos0;
  a.logits_each = logits_each ? 1 : 0;
  a.logits = logits ? e->d_logits : nullptr;
  a.argmax_out = e->d_argmax;
  if (n > 1 && e->lwe_ok) {
    CUDA_TRY(e, cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream));
    int f = 0;
    TRY(lwe_run(e, slot, e->d_ids, n, pos0, logits_each, logits ? e->d_logits : nullptr, e->d_argmax, &f));
  } else {
    TRY(launch(e, a, (n + e->mmax - 1) / e->mmax, n > 1));
  }
  TRY(fetch_status(e));
  if (logits) CUDA_TRY(e, cudaMemcpyAsync(logits, e->d_logits, need * 4, cudaMemcpyDeviceToHost, e->stream));
  if (argmax)
    CUDA_TRY(e, cudaMemcpyAsync(argmax, e->d_argmax, (logits_each ? n : 1) * 4, cudaMemcpyDeviceToHost, e->stream));
  TRY(finish(e));
  s.cache_len = pos0 + n;
  return MLLM_OK;
}

int mllm_generate(mllm_engine* e, int slot, const int32_t* ids, int n, int max_new, int32_t eos, int spec_k, int ngram,
                  int32_t* out_ids, mllm_stats* st) {
  if (!e) return MLLM_ERR_ARG;
  cudaSetDevice(e->device);
  if (!ids || !out_ids) return fail(e, MLLM_ERR_ARG, "null ids/out_ids");
  if (max_new <= 0) return fail(e, MLLM_ERR_ARG, "max_new must be positive");
  // engine/infer.js:604-608
  const int max_prompt = std::max(1, e->md.max_seq - max_new - 1);
  if (n > max_prompt) {
    ids += n - max_prompt;
    n = max_prompt;
  }
  if (n <= 0) return fail(e, MLLM_ERR_ARG, "empty prompt");
  if (n > e->md.kv_len - 1) return fail(e, MLLM_ERR_ARG, "prompt of %d ids does not fit the cache", n);
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= e->md.vocab) return fail(e, MLLM_ERR_ARG, "token id %d out of range", ids[i]);
  if (max_new > e->md.kv_len + 16) return fail(e, MLLM_ERR_ARG, "max_new exceeds the cache length");
  CUDA_TRY(e, cudaMemcpyAsync(e->d_ids, ids, n * 4, cudaMemcpyHostToDevice, e->stream));
  TRY(generate_impl(e, slot, e->d_ids, n, max_new, eos, spec_k, ngram, e->d_out, st));
  const int gen = e->h_status[ST_NGEN];
  CUDA_TRY(e, cudaMemcpyAsync(out_ids, e->d_out, std::max(gen, 0) * 4, cudaMemcpyDeviceToHost, e->stream));
  CUDA_TRY(e, cudaStreamSynchronize(e->stream));
  return MLLM_OK;
}

int mllm_generate_stream(mllm_engine* e, int slot, const int32_t* ids, int n, int max_new, int32_t eos, int spec_k,
                         int ngram, int32_t* out_ids, mllm_stats* st, mllm_token_fn on_token, void* user) {
  if (!e) return MLLM_ERR_ARG;
  if (!on_token) return mllm_generate(e, slot, ids, n, max_new, eos, spec_k, ngram, out_ids, st);
  cudaSetDevice(e->device);
  *reinterpret_cast<volatile int32_t*>(e->h_stream) = 0;  // no kernel of this handle is running
  e->on_token = on_token;
  e->on_token_user = user;
  e->delivered = 0;
  const int rc = mllm_generate(e, slot, ids, n, max_new, eos, spec_k, ngram, out_ids, st);
  // ids of a path that does not publish (the persistent multi-token kernel) go out after the launch
  if (rc == MLLM_OK)
    for (int i = e->delivered; i < e->h_status[ST_NGEN]; ++i) on_token(out_ids[i], i, i == 0 ? 0 : 1, user);
  e->on_token = nullptr;
  e->on_token_user = nullptr;
  return rc;
}

int mllm_selftest_timeout(mllm_engine* e, int wait_ms) {
  if (!e || wait_ms <= 0) return MLLM_ERR_ARG;
  cudaSetDevice(e->device);
  RunArgs a{};
  a.kc = e->slots[0].k;
  a.vc = e->slots[0].v;
  a.mode = MODE_SELFTEST_WAIT;
  a.wait_ns = (uint64_t)wait_ms * 1000000ull;
  TRY(launch(e, a, 1, false));
  TRY(fetch_status(e));
  return finish(e);
}

int mllm_generate_device(mllm_engine* e, int slot, const int32_t* d_ids, int n, int max_new, int32_t eos, int spec_k,
                         int ngram, int32_t* d_out, mllm_stats* st) {
  if (!e) return MLLM_ERR_ARG;
  cudaSetDevice(e->device);
  if (!d_ids || !d_out) return fail(e, MLLM_ERR_ARG, "null device pointers");
  if (n <= 0 || n > std::max(1, e->md.max_seq - max_new - 1) || n > e->md.kv_len - 1)
    return fail(e, MLLM_ERR_ARG, "prompt length %d does not fit (truncate on the host first)", n);
  return generate_impl(e, slot, d_ids, n, max_new, eos, spec_k, ngram, d_out, st);
}


// Replicated multi-sequence greedy decode (see include/mllm.h).  Host side: truncation and the
// prefill plan; device side: token-batch prefill forwards, first ids, then one batched decode step
// per generated position, captured once as a CUDA graph and replayed.
int mllm_generate_batch(mllm_engine* e, int n_seq, const int32_t* ids, const int32_t* offsets, int max_new,
                        int32_t eos, int32_t* out_ids, int32_t* n_out, int32_t* stop, mllm_batch_stats* stats) {
  if (!e) return MLLM_ERR_ARG;
  cudaSetDevice(e->device);
  if (!ids || !offsets || !out_ids || !n_out) return fail(e, MLLM_ERR_ARG, "null ids/offsets/out_ids/n_out");
  if (n_seq <= 0 || n_seq > (int)e->slots.size())
    return fail(e, MLLM_ERR_ARG, "n_seq %d outside [1, %zu] (max_slots)", n_seq, e->slots.size());
  if (n_seq > e->tmax) return fail(e, MLLM_ERR_UNSUPPORTED, "n_seq %d exceeds %d rows per forward", n_seq, e->tmax);
  if (!e->lwe_ok) return fail(e, MLLM_ERR_UNSUPPORTED, "nHeads / nKvHeads above %d", kLweMaxRep);
  if (max_new <= 0 || max_new > e->md.kv_len + 16) return fail(e, MLLM_ERR_ARG, "max_new outside [1, kv_len + 16]");
  const ModelDev& md = e->md;
  const int kv_len = md.kv_len;
  // engine/infer.js:604-608 per sequence
  const int max_prompt = std::max(1, md.max_seq - max_new - 1);
  std::vector<int32_t> lens(n_seq), first(n_seq);
  for (int q = 0; q < n_seq; ++q) {
    const int len = offsets[q + 1] - offsets[q];
    if (offsets[q] < 0 || len <= 0) return fail(e, MLLM_ERR_ARG, "sequence %d has an empty prompt", q);
    const int tl = std::min(len, max_prompt);
    if (tl > kv_len - 1) return fail(e, MLLM_ERR_ARG, "prompt of sequence %d does not fit the cache", q);
    lens[q] = tl;
    first[q] = offsets[q] + (len - tl);
  }
  const int total_ids = offsets[n_seq];
  const long l0 = launches_now(e);
  long graph_kernels = 0;  // kernels per decode step (one graph launch each)
  for (int i = offsets[0]; i < total_ids; ++i)
    if (ids[i] < 0 || ids[i] >= md.vocab) return fail(e, MLLM_ERR_ARG, "token id %d out of range", ids[i]);
  // Plan: every prompt token (slot, position, source index); forward c takes tokens [c*tmax, ..).
  // Per forward, the lm rows are the tokens that end a prompt.
  std::vector<int32_t> p_slot, p_pos, p_src, lm_src, lm_slot, lm_off{0};
  for (int q = 0; q < n_seq; ++q)
    for (int i = 0; i < lens[q]; ++i) {
      p_slot.push_back(q);
      p_pos.push_back(i);
      p_src.push_back(first[q] + i);
    }
  const int P = (int)p_slot.size();
  const int nchunk = (P + e->tmax - 1) / e->tmax;
  for (int c = 0; c < nchunk; ++c) {
    const int c0 = c * e->tmax, c1 = std::min(P, c0 + e->tmax);
    for (int k = c0; k < c1; ++k)
      if (p_pos[k] == lens[p_slot[k]] - 1) {
        lm_src.push_back(k - c0);
        lm_slot.push_back(p_slot[k]);
      }
    lm_off.push_back((int)lm_src.size());
  }
  // one device buffer: slot[P] pos[P] src[P] lm_src[n] lm_slot[n]
  std::vector<int32_t> plan;
  plan.reserve(3 * P + 2 * n_seq);
  plan.insert(plan.end(), p_slot.begin(), p_slot.end());
  plan.insert(plan.end(), p_pos.begin(), p_pos.end());
  plan.insert(plan.end(), p_src.begin(), p_src.end());
  plan.insert(plan.end(), lm_src.begin(), lm_src.end());
  plan.insert(plan.end(), lm_slot.begin(), lm_slot.end());
  const size_t state_words = 2 * (size_t)n_seq + 16;  // counts[n], lens[n], active
  TRY(grow(e, e->g_bids, (size_t)total_ids * 4));
  TRY(grow(e, e->g_plan, plan.size() * 4));
  TRY(grow(e, e->g_bout, (size_t)n_seq * max_new * 4));
  TRY(grow(e, e->g_state, state_words * 4));
  const bool gpt2 = md.arch == 1;
  if (gpt2) TRY(grow(e, e->g_blogits, (size_t)n_seq * md.vocab * 4));
  int32_t* d_bids = (int32_t*)e->g_bids.p;
  int32_t* d_plan = (int32_t*)e->g_plan.p;
  int32_t* d_bout = (int32_t*)e->g_bout.p;
  int32_t* d_counts = (int32_t*)e->g_state.p;
  int32_t* d_lens = d_counts + n_seq;
  int32_t* d_active = d_lens + n_seq;
  float* d_blogits = (float*)e->g_blogits.p;
  cudaStream_t st = e->stream;
  CUDA_TRY(e, cudaMemcpyAsync(d_bids, ids, (size_t)total_ids * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(e, cudaMemcpyAsync(d_plan, plan.data(), plan.size() * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(e, cudaMemcpyAsync(d_lens, lens.data(), (size_t)n_seq * 4, cudaMemcpyHostToDevice, st));
  CUDA_TRY(e, cudaMemsetAsync(e->d_err, 0, sizeof(int), st));
  CUDA_TRY(e, cudaMemsetAsync(e->d_status, 0, ST_WORDS * sizeof(int32_t), st));
  lwe_mark_time(e->d_status, ST_T0, st);
  // ---- prefill
  const int32_t* d_pslot = d_plan;
  const int32_t* d_ppos = d_plan + P;
  const int32_t* d_psrc = d_plan + 2 * P;
  const int32_t* d_lmsrc = d_plan + 3 * P;
  const int32_t* d_lmslot = d_lmsrc + n_seq;
  const LweArgs base = lwe_args(e);
  for (int c = 0; c < nchunk; ++c) {
    const int c0 = c * e->tmax, Tc = std::min(e->tmax, P - c0);
    const int nlm = lm_off[c + 1] - lm_off[c];
    LweArgs a = base;
    a.slot = const_cast<int32_t*>(d_pslot + c0);
    a.pos = const_cast<int32_t*>(d_ppos + c0);
    a.lm_src = const_cast<int32_t*>(d_lmsrc + lm_off[c]);
    lwe_gather(a.tok, d_bids, d_psrc + c0, Tc, st);
    CUDA_TRY(e, lwe_forward(a, e->lh, Tc, nlm, true, nullptr, false, st));
    if (nlm) lwe_batch_first(a.amax, d_lmslot + lm_off[c], nlm, max_new, eos, kv_len, d_bout, d_counts, d_lens, st);
  }
  lwe_mark_time(e->d_status, ST_TFIRST, st);
  // ---- decode: row t = sequence t
  int steps_max = 0;
  for (int q = 0; q < n_seq; ++q) steps_max = std::max(steps_max, std::min(max_new, kv_len - lens[q]) - 1);
  int steps = 0;
  if (steps_max > 0) {
    const LweArgs d = base;  // tok/slot/pos/lm_src: the engine's own rows
    lwe_batch_decode_setup(d, n_seq, d_bout, d_counts, d_lens, max_new, st);
    auto step = [&]() -> cudaError_t {
      cudaError_t r = lwe_forward(d, e->lh, n_seq, n_seq, false, gpt2 ? d_blogits : nullptr, true, st);
      if (r != cudaSuccess) return r;
      if (gpt2) lwe_penalised_argmax(d_blogits, md.vocab, n_seq, d_bout, d_counts, max_new, d.amax, st);
      lwe_batch_advance(d, n_seq, max_new, eos, d_bout, d_counts, d_lens, st);
      return cudaGetLastError();
    };
    cudaGraphExec_t exec = nullptr;
    if (e->lwe_graph) {
      cudaGraph_t graph = nullptr;
      CUDA_TRY(e, cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
      const long c0 = launches_now(e);
      const cudaError_t r1 = step();
      graph_kernels = launches_now(e) - c0;  // captured, not run
      const cudaError_t r2 = cudaStreamEndCapture(st, &graph);
      if (r1 != cudaSuccess || r2 != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return fail(e, MLLM_ERR_CUDA, "capture of the decode step failed: %s",
                    cudaGetErrorString(r1 != cudaSuccess ? r1 : r2));
      }
      const cudaError_t r3 = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      if (r3 != cudaSuccess) return fail(e, MLLM_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(r3));
    }
    // With an EOS id the batch may finish early: every 16 steps the number of running sequences is
    // read back (the steps already queued behind it keep the GPU busy meanwhile).
    cudaError_t rs = cudaSuccess;
    for (; steps < steps_max && rs == cudaSuccess; ++steps) {
      rs = exec ? cudaGraphLaunch(exec, st) : step();
      if (eos >= 0 && rs == cudaSuccess && (steps & 15) == 15 && steps + 1 < steps_max) {
        lwe_count_active(d_counts, n_seq, d_active, st);
        rs = cudaMemcpyAsync(e->h_active, d_active, 4, cudaMemcpyDeviceToHost, st);
        if (rs == cudaSuccess) rs = cudaStreamSynchronize(st);
        if (rs == cudaSuccess && *e->h_active == 0) {
          ++steps;
          break;
        }
      }
    }
    if (exec) cudaGraphExecDestroy(exec);
    if (rs != cudaSuccess) return fail(e, MLLM_ERR_CUDA, "batched decode step: %s", cudaGetErrorString(rs));
  }
  lwe_mark_time(e->d_status, ST_TEND, st);
  std::vector<int32_t> counts(n_seq);
  CUDA_TRY(e, cudaMemcpyAsync(out_ids, d_bout, (size_t)n_seq * max_new * 4, cudaMemcpyDeviceToHost, st));
  CUDA_TRY(e, cudaMemcpyAsync(counts.data(), d_counts, (size_t)n_seq * 4, cudaMemcpyDeviceToHost, st));
  TRY(fetch_status(e));
  TRY(finish(e));
  int total = 0;
  for (int q = 0; q < n_seq; ++q) {
    const int c = std::abs(counts[q]);
    n_out[q] = c;
    total += c;
    if (stop) stop[q] = (c > 0 && out_ids[(size_t)q * max_new + c - 1] == eos) ? MLLM_STOP_EOS : MLLM_STOP_MAX_NEW;
    e->slots[q].cache_len = std::min(lens[q] + c - 1, kv_len);
  }
  if (stats) {
    const int32_t* hs = e->h_status;
    stats->n_seq = n_seq;
    stats->total_generated = total;
    stats->steps = steps;
    stats->prefill_forwards = nchunk;
    const uint64_t t0 = u64_at(hs, ST_T0), t1 = u64_at(hs, ST_TFIRST), t2 = u64_at(hs, ST_TEND);
    stats->prefill_ms = t1 > t0 ? (float)((t1 - t0) * 1e-6) : 0.f;
    stats->total_ms = t2 > t0 ? (float)((t2 - t0) * 1e-6) : 0.f;
    // a graph launch runs graph_kernels kernels; the capture itself ran none
    stats->kernel_launches = (int32_t)(launches_now(e) - l0 - graph_kernels + graph_kernels * (long)steps);
  }
  return MLLM_OK;
}

}  // extern "C"
