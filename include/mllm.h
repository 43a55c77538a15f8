/*
 * mllm.h — C ABI of the B200 Q4 decode backend for MicroLLM lab (libmllm_cuda.so).
 *
 * Plain pointers and sizes only.  Every entry point returns an mllm_status code; a message for the
 * last failure is available from mllm_last_error(handle) (or mllm_last_error(NULL) for failures that
 * happen before a handle exists).  The library never falls back to a CPU path: with no usable CUDA
 * device mllm_create fails with MLLM_ERR_CUDA.
 *
 * Each entry point names the reference interface it replaces (paths relative to the reference
 * project root).  The JavaScript engine surface those bind to is PetitGPT (engine/infer.js:289-647)
 * and GpuPetitGPT (engine/webgpu.js:867-1297); a Node-API addon binds each entry point one to one.
 */
#ifndef MLLM_H
#define MLLM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mllm_engine mllm_engine;

typedef enum {
  MLLM_OK = 0,
  MLLM_ERR_FORMAT = -1,      /* bad magic, truncated file, malformed tensor table */
  MLLM_ERR_UNSUPPORTED = -2, /* dtype other than q4, head_dim != 64, shape beyond the kernel limits */
  MLLM_ERR_ARG = -3,         /* token id out of range, position beyond maxSeqLen, bad slot, null pointer */
  MLLM_ERR_OOM = -4,         /* device allocation failed */
  MLLM_ERR_CUDA = -5,        /* CUDA runtime error (no device, launch failure, ...) */
  MLLM_ERR_TIMEOUT = -6      /* a device-side wait ran out its time limit; the handle stays usable */
} mllm_status;

typedef enum { MLLM_STOP_EOS = 0, MLLM_STOP_MAX_NEW = 1, MLLM_STOP_CONTEXT = 2 } mllm_stop;

/* PGW1 storage kinds: the dtype byte of the header and each tensor's storage (engine/weights.js:3). */
typedef enum { MLLM_DTYPE_F32 = 0, MLLM_DTYPE_F16 = 1, MLLM_DTYPE_BF16 = 2, MLLM_DTYPE_Q8 = 3, MLLM_DTYPE_Q4 = 4 } mllm_dtype;

/* Result of a generate call: engine/infer.js:617-645 and engine/webgpu.js:1272-1281. */
typedef struct {
  int32_t n_generated;  /* ids written to out_ids */
  int32_t stop_reason;  /* mllm_stop */
  int32_t spec_hits;    /* accepted draft tokens (specHits) */
  int32_t spec_tries;   /* speculation iterations, each one verify forward, drafted or not (specTries) */
  int32_t forwards;     /* forward passes run on the device, prefill chunks included */
  int32_t prompt_len;   /* prompt length after truncation (engine/infer.js:604-608) */
  float ttft_ms;        /* device time from launch to the first generated id */
  float total_ms;       /* device time of the whole call */
  int32_t kernel_launches; /* CUDA kernels the call launched */
} mllm_stats;

/*
 * Load a PGW1 Q4 file and upload it to `device`.  Replaces parsePgw + new PetitGPT(bundle)
 * (engine/weights.js:5-40, engine/infer.js:290-311) and GpuPetitGPT.init (engine/webgpu.js:892-1106).
 * The buffer is only borrowed for the call.  `max_slots` independent sequences (KV caches) are
 * allocated; `kv_len` caps each cache's positions (0 = the file's maxSeqLen).
 */
int mllm_create(int device, const uint8_t* pgw, size_t len, int max_slots, int kv_len, mllm_engine** out);

/* engine/webgpu.js:1284-1297 (destroy). */
void mllm_destroy(mllm_engine* e);

/* Message of the last failure on this handle, or of the last failed mllm_create when e is NULL. */
const char* mllm_last_error(const mllm_engine* e);

/*
 * Model configuration as parsed from the header (engine/weights.js:17-29):
 * cfg[0..9] = arch (0 llama, 1 gpt2), vocabSize, nLayers, dModel, nHeads, nKvHeads, dFf, maxSeqLen,
 * kv_len, max_tokens_per_forward.
 */
int mllm_config(const mllm_engine* e, int32_t* cfg10);

/*
 * Launch on the caller's CUDA stream (a cudaStream_t; NULL restores the handle's own stream).  The
 * reference engine submits to its WebGPU device queue (engine/webgpu.js:1120-1138); this is the
 * equivalent hook, so that callers can order, overlap and time the launches with their own events.
 */
int mllm_set_stream(mllm_engine* e, void* stream);

/* Device bytes held by the handle (GpuPetitGPT.bytesAllocated, engine/webgpu.js:1047-1065). */
size_t mllm_bytes_allocated(const mllm_engine* e);

/*
 * The kernel that runs single-token decode on this handle ("decode1: grid of G CTAs" or
 * "cdec_kernel: N cluster(s) of 16 CTAs").  No reference counterpart: the reference has one WebGPU
 * pipeline per stage (engine/webgpu.js:892-1106); this names the launch that replaces them.
 */
const char* mllm_decode_kernel(const mllm_engine* e);

/* engine/infer.js:348-358 (resetCache) for one slot. */
int mllm_reset(mllm_engine* e, int slot);

/* engine/infer.js:357 (cacheLen) for one slot. */
int mllm_cache_len(const mllm_engine* e, int slot);

/*
 * One forward over n host token ids at positions pos0 .. pos0+n-1 of `slot`, writing their K/V into
 * the slot's cache and setting cacheLen = pos0 + n.  forwardPrompt(ids) is pos0 = 0
 * (engine/infer.js:553-577); forwardDecode(id) is n = 1, pos0 = cacheLen (engine/infer.js:579-601);
 * logits_each = 1 is the verify forward of engine/webgpu.js:1248 (one logits row per token).
 * logits (nullable, host): [vocab] for the last token, or [n][vocab] when logits_each.
 * argmax (nullable, host): greedy ids per returned logits row (engine/infer.js:240-250, lowest index
 * on ties).
 */
int mllm_forward(mllm_engine* e, int slot, const int32_t* ids, int n, int pos0, int logits_each, float* logits,
                 int32_t* argmax);

/*
 * Whole greedy generation in one device launch: engine/infer.js:603-646 when spec_k == 0, and the
 * fused path with prompt-lookup speculation of engine/webgpu.js:1164-1282 (lookupDraft
 * engine/webgpu.js:846-865) when spec_k > 0 (n-gram size `ngram`).  GPT-2 files use the penalised
 * argmax of engine/infer.js:252-287.  eos = -1 disables the EOS stop.  ids/out_ids are host arrays;
 * out_ids has room for max_new ids.  stats (nullable) receives the counters.
 */
int mllm_generate(mllm_engine* e, int slot, const int32_t* ids, int n, int max_new, int32_t eos, int spec_k,
                  int ngram, int32_t* out_ids, mllm_stats* stats);

/*
 * Streaming form of mllm_generate: the same call, with each generated id handed to
 * on_token(id, index, phase, user) on the calling thread while the device is still generating
 * (engine/infer.js:615,630 and engine/webgpu.js:1202-1237, 1253, 1265 call onToken per id; phase 0 =
 * "prefill" (the first id), 1 = "decode", 2 = "spec" (an accepted draft id)).  The kernels publish
 * every id into mapped pinned host memory with a system-scope release as soon as it is chosen; the
 * call polls those words while it waits for the device, so no per-token synchronisation is added.
 * Ids arrive in generation order, each exactly once; out_ids and stats are filled as by
 * mllm_generate.  on_token must not call back into this handle.  NULL on_token = mllm_generate.
 */
typedef void (*mllm_token_fn)(int32_t id, int32_t index, int32_t phase, void* user);
int mllm_generate_stream(mllm_engine* e, int slot, const int32_t* ids, int n, int max_new, int32_t eos, int spec_k,
                         int ngram, int32_t* out_ids, mllm_stats* stats, mllm_token_fn on_token, void* user);

/* mllm_generate with the prompt and the output already in device memory (d_ids: int32 [n],
 * d_out: int32 [max_new]); stats stay host-side.  Used to time the device path without copies. */
int mllm_generate_device(mllm_engine* e, int slot, const int32_t* d_ids, int n, int max_new, int32_t eos,
                         int spec_k, int ngram, int32_t* d_out, mllm_stats* stats);

/* Result of a batched generate call. */
typedef struct {
  int32_t n_seq;            /* sequences run */
  int32_t total_generated;  /* ids generated over all sequences */
  int32_t steps;            /* batched decode steps after the prefill */
  int32_t prefill_forwards; /* token-batch forwards of the prefill */
  float prefill_ms;         /* device time of the prefill (all prompts, first ids) */
  float total_ms;           /* device time of the whole call */
  int32_t kernel_launches;  /* CUDA kernels the call ran (graph nodes counted per replay) */
} mllm_batch_stats;

/*
 * Replicated multi-sequence greedy decode: n_seq independent prompts run as one batch, sequence s on
 * slot s (n_seq <= max_slots and <= max_tokens_per_forward).  Each sequence follows
 * engine/infer.js:603-646 exactly as mllm_generate would (its own truncation, first id from its
 * prefill, EOS / max_new / cache-length stops; GPT-2 files use the penalised argmax of
 * engine/infer.js:252-287 over that sequence's own generated ids), so the output per sequence is
 * identical to n_seq separate mllm_generate calls.  The reference runs one sequence per engine
 * (engine/worker.js:149-159); this is the batched form of that loop (generateBatch in the JS
 * binding).  Prompts: ids[offsets[s] .. offsets[s+1]) (host, offsets has n_seq + 1 entries).
 * Output: out_ids [n_seq][max_new] (host), n_out [n_seq] ids generated per sequence, stop
 * [n_seq] (nullable) mllm_stop per sequence.  Prefill and decode run as token-batch forwards
 * on the tensor cores; each decode step is one CUDA graph launch.
 */
int mllm_generate_batch(mllm_engine* e, int n_seq, const int32_t* ids, const int32_t* offsets, int max_new,
                        int32_t eos, int32_t* out_ids, int32_t* n_out, int32_t* stop, mllm_batch_stats* stats);

/*
 * Failure-detection self-test (no counterpart in the reference): launches the decode kernel in a
 * mode where every CTA waits for a word that nothing writes, with a `wait_ms` limit.  Expected
 * result: MLLM_ERR_TIMEOUT, after which the handle keeps working.  Nothing faults or traps.
 */
int mllm_selftest_timeout(mllm_engine* e, int wait_ms);

/*
 * Q4 group-32 matrix-vector / skinny-matrix product y[m][r] = sum_g sc[r][g] * sum_k (q[r][32g+k]-8) x[m][32g+k]
 * for m < n_act (engine/infer.js:88-116, engine/kernels.rs:60-97) on device pointers in the PGW
 * layout: packed [rows][cols/2] bytes, scales [rows][cols/32] f32, x [n_act][cols], y [n_act][rows].
 * fp32 accumulation.  n_act <= 16.  stream is a cudaStream_t (NULL = the device's default stream).
 */
int mllm_gemv_q4(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y, int rows, int cols,
                 int n_act, void* stream);

/*
 * Matrix-vector / skinny-matrix product for the other PGW storage kinds: gemvF32, gemvF16, gemvBf16
 * and gemvQ8 (engine/infer.js:10-86, bound per tensor storage at engine/infer.js:314-345).
 * y[m][r] = sum_k W[r][k] x[m][k] for m < n_act, with W in storage `dtype` on the device: f32
 * [rows][cols]; f16 or bf16 as 16-bit words [rows][cols]; q8 as int8 [rows][cols] with d_scales f32
 * [rows], applied after the row sum as gemvQ8 does (d_scales is ignored for the other kinds).
 * fp32 accumulation.  n_act <= 16; a row must be whole 16-byte chunks (cols x element bytes a multiple
 * of 16, cols a multiple of 4) and d_w, d_x 16-byte aligned, else MLLM_ERR_ARG.  MLLM_DTYPE_Q4 returns
 * MLLM_ERR_UNSUPPORTED: its packed layout goes to mllm_gemv_q4.
 */
int mllm_gemv(int dtype, const void* d_w, const float* d_scales, const float* d_x, float* d_y, int rows, int cols,
              int n_act, void* stream);

/*
 * The same product for any number of activation rows on the tensor cores: n_act >= 1 rows of f32
 * activations x [n_act][cols] -> y [n_act][rows].  Each activation is split into fp16 hi + lo halves
 * (relative residual <= 2^-22) that multiply the dequantised (q - 8) weights (exact in fp16) with
 * fp32 accumulation; group scales are applied in fp32.  The fp16 halves live in a per-device
 * workspace that this call allocates on first use (and grows when a larger call arrives; a replaced
 * workspace is kept until exit, since kernels enqueued earlier may still read it).  All calls on one
 * device share that workspace: calls whose kernels overlap on the GPU (different streams or host
 * threads) race on it and must be serialised by the caller.
 * Replaces gemmGeneric (engine/infer.js:118-132: a row loop of gemvQ4) for prefill, verify and
 * multi-sequence decode.
 */
int mllm_gemm_q4(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y, int rows, int cols,
                 int n_act, void* stream);

/*
 * Allocation-free form of mllm_gemm_q4 (no counterpart in the reference).  For callers that cannot
 * call cudaMalloc — a host runtime that owns all device memory through its own pool, or a
 * latency-sensitive thread that cannot take cudaMalloc's implicit synchronisation — the fp16
 * scratch lives in a fixed 4 MiB array inside the library (held by every device that loads it, until
 * exit), so no call allocates or frees anything.  Limit: n_act * cols <= 1,048,576 activation values;
 * larger calls return MLLM_ERR_ARG with a message in mllm_last_error(NULL).  The first call on a
 * device looks up the array's device address with that device current, so make the first call
 * before any stream capture.  All calls share the array: calls that overlap on the GPU (different
 * streams, different host threads) race on it and must be serialised by the caller.
 */
int mllm_gemm_q4_noalloc(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y, int rows,
                         int cols, int n_act, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLLM_H */
