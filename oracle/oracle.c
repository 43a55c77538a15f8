/*
 * oracle.c — CPU restatement of MicroLLM lab's Q4 decode path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity checker for the CUDA product in microllm-lab_b200/.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs may load it.
 * The product never links it and has no CPU fallback.
 *
 * What it restates (paths relative to the reference project root):
 *   engine/infer.js:88-116    gemvQ4            f64 accumulation, 4-byte unroll order b0..b3
 *   engine/infer.js:134-143   rmsNorm           eps 1e-6, f64 sum of squares
 *   engine/infer.js:147-164   layerNorm         eps 1e-5, [gain; bias] packed
 *   engine/infer.js:166-171   geluNewInPlace    tanh form
 *   engine/infer.js:178-183   siluMul
 *   engine/infer.js:185-225   buildRope/applyRope  f32-rounded inverse frequencies
 *   engine/infer.js:227-238   softmaxInPlace    f64 sum of unrounded exps, f32 store
 *   engine/infer.js:240-287   argmax / argmaxGpt2
 *   engine/infer.js:360-420   embed / _embedRowQuant (tied lm_head row, GPT-2 scale_factors + wpe)
 *   engine/infer.js:422-527   attention / ffn   (generalised to t tokens at pastLen, as the code allows)
 *   engine/infer.js:553-646   forwardPrompt / forwardDecode / generate
 *   engine/webgpu.js:846-865  lookupDraft       prompt-lookup n-gram draft
 *   engine/webgpu.js:1164-1282 generate (fused path with speculation: verify forward + greedy accept)
 *   engine/kernels.rs:60-97   gemv_q4           f32 accumulation variant (second GEMV reference)
 *
 * Numeric rules: JavaScript numbers are IEEE f64, typed-array stores round to f32.  Every
 * `let s = 0` accumulator is a double here, every Float32Array store is a (float) cast, and
 * expressions are evaluated in the same order as the JS source.  Build with -ffp-contract=off and
 * without fast-math so that no FMA contraction or reassociation changes a rounding.
 *
 * Parity pinning: the JS source cannot be executed on this machine (no JavaScript runtime).  The
 * Q4 pack and PGW1 container are pinned against the reference's own Python converter
 * (tools/convert_hf_to_pgw.py) run here; the forward math is pinned against HF transformers'
 * Llama forward on the dequantised weights in float64, the graph infer.js:1-4 states it matches.
 */
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define EPS 1e-6    /* engine/infer.js:8 */
#define LN_EPS 1e-5 /* engine/infer.js:145 */

/* PGW1 storage kinds (engine/weights.js:3) */
enum { ST_F32 = 0, ST_F16 = 1, ST_BF16 = 2, ST_Q8 = 3, ST_Q4 = 4 };

typedef struct {
  char name[64];
  int storage; /* ST_* */
  int rows, cols, group;
  const uint8_t* data;   /* f32 values, 16-bit words (f16 / bf16), int8 (q8) or q4 packed bytes */
  const float* scale;    /* q8: one per row; q4: one per group */
} otensor;

typedef struct {
  int arch; /* 0 llama, 1 gpt2 */
  int vocab, n_layers, d_model, n_heads, n_kv_heads, d_ff, max_seq;
  double rope_theta, rope_pct;
} ocfg;

typedef struct opool opool;

typedef struct oracle_model {
  ocfg c;
  int head_dim, kv_dim, rep;
  int n_tensors;
  otensor* tensors;
  /* bound tensors */
  const otensor* lm_head;
  const otensor** qkv; const otensor** proj; const otensor** w1; const otensor** w3; const otensor** w2;
  const float** norm1; const float** norm2;
  const float** qkv_b; const float** proj_b; const float** fc_b; const float** mproj_b;
  const float* norm_f; const float* wpe; const float* scale_factors;
  /* rope tables */
  int rope_dim;
  float* rope_cos; float* rope_sin;
  /* KV cache: per layer [nKv][maxSeq][hd] */
  float** k_cache; float** v_cache;
  int cache_len;
  int threads;
  opool* pool;
} oracle_model;

/* ------------------------------------------------------------------------------------------ */
/* GEMV kernels                                                                               */
/* ------------------------------------------------------------------------------------------ */

/* engine/infer.js:88-116 */
static void gemv_q4_row(int n, const uint8_t* row, const float* so, int group, const float* x, float* y) {
  const int ng = n / group, halfGroup = group / 2;
  double acc = 0;
  for (int g = 0; g < ng; g++) {
    const double sc = so[g];
    const uint8_t* base = row + g * halfGroup;
    const float* xb = x + g * group;
    double s = 0;
    for (int k = 0; k < halfGroup; k += 4) {
      const int b0 = base[k], b1 = base[k + 1], b2 = base[k + 2], b3 = base[k + 3];
      const float* xi = xb + k * 2;
      double t = (double)((b0 & 15) - 8) * xi[0];
      t += (double)((b0 >> 4) - 8) * xi[1];
      t += (double)((b1 & 15) - 8) * xi[2];
      t += (double)((b1 >> 4) - 8) * xi[3];
      t += (double)((b2 & 15) - 8) * xi[4];
      t += (double)((b2 >> 4) - 8) * xi[5];
      t += (double)((b3 & 15) - 8) * xi[6];
      t += (double)((b3 >> 4) - 8) * xi[7];
      s += t;
    }
    acc += s * sc;
  }
  *y = (float)acc;
}

/*
 * A small spinning thread pool splits GEMV rows across host cores for the all-cores CPU baseline.
 * Rows are independent, so the thread count never changes a result.
 */
typedef struct {
  int m, n, group;
  const uint8_t* packed;
  const float* scale;
  const float* x;
  float* y;
} gemv_job;

struct opool {
  pthread_t th[256];
  int nthreads; /* workers + the calling thread */
  atomic_int gen, done, stop;
  gemv_job job;
};

static void gemv_slice(const gemv_job* j, int part, int nparts) {
  const int ng = j->n / j->group;
  const size_t packedRow = (size_t)j->n / 2;
  const int lo = (int)((long)j->m * part / nparts), hi = (int)((long)j->m * (part + 1) / nparts);
  for (int i = lo; i < hi; i++)
    gemv_q4_row(j->n, j->packed + (size_t)i * packedRow, j->scale + (size_t)i * ng, j->group, j->x, j->y + i);
}

typedef struct {
  opool* p;
  int idx;
} worker_arg;

static void* pool_worker(void* a) {
  worker_arg* wa = (worker_arg*)a;
  opool* p = wa->p;
  const int idx = wa->idx;
  free(wa);
  int seen = 0;
  for (;;) {
    int g, spins = 0;
    while ((g = atomic_load_explicit(&p->gen, memory_order_acquire)) == seen) {
      if (atomic_load_explicit(&p->stop, memory_order_relaxed)) return NULL;
      if (++spins > 2000) {
        sched_yield();
        spins = 0;
      }
    }
    seen = g;
    gemv_slice(&p->job, idx, p->nthreads);
    atomic_fetch_add_explicit(&p->done, 1, memory_order_release);
  }
}

static opool* pool_create(int nthreads) {
  opool* p = (opool*)calloc(1, sizeof(opool));
  if (nthreads > 256) nthreads = 256;
  p->nthreads = nthreads;
  for (int i = 1; i < nthreads; i++) {
    worker_arg* wa = (worker_arg*)malloc(sizeof(worker_arg));
    wa->p = p;
    wa->idx = i;
    pthread_create(&p->th[i], NULL, pool_worker, wa);
  }
  return p;
}

static void pool_destroy(opool* p) {
  if (!p) return;
  atomic_store(&p->stop, 1);
  for (int i = 1; i < p->nthreads; i++) pthread_join(p->th[i], NULL);
  free(p);
}

static void pool_gemv(opool* p, const gemv_job* j) {
  p->job = *j;
  atomic_store_explicit(&p->done, 0, memory_order_relaxed);
  atomic_fetch_add_explicit(&p->gen, 1, memory_order_release);
  gemv_slice(j, 0, p->nthreads);
  int spins = 0;
  while (atomic_load_explicit(&p->done, memory_order_acquire) < p->nthreads - 1)
    if (++spins > 2000) {
      sched_yield();
      spins = 0;
    }
}

static void gemv_q4_pool(opool* pool, int m, int n, const uint8_t* packed, const float* scale, int group,
                         const float* x, float* y) {
  gemv_job j = {m, n, group, packed, scale, x, y};
  if (pool && (long)m * n >= 65536) pool_gemv(pool, &j);
  else gemv_slice(&j, 0, 1);
}

void oracle_gemv_q4(int m, int n, const uint8_t* packed, const float* scale, int group, const float* x,
                    float* y, int threads) {
  opool* p = threads > 1 ? pool_create(threads) : NULL;
  gemv_q4_pool(p, m, n, packed, scale, group, x, y);
  pool_destroy(p);
}

/* engine/kernels.rs:60-97 — f32 accumulation, element order lo then hi nibble */
void oracle_gemv_q4_f32acc(int m, int n, const uint8_t* packed, const float* scale, int group, const float* x,
                           float* y) {
  const int ng = n / group;
  const size_t packedRow = (size_t)n / 2;
  for (int i = 0; i < m; i++) {
    float acc = 0.0f;
    const uint8_t* row = packed + (size_t)i * packedRow;
    for (int g = 0; g < ng; g++) {
      const float sc = scale[(size_t)i * ng + g];
      const uint8_t* base = row + g * (group / 2);
      float s = 0.0f;
      for (int k = 0; k < group; k += 2) {
        const uint8_t b = base[k / 2];
        s += (float)((int)(b & 15) - 8) * x[g * group + k];
        s += (float)((int)(b >> 4) - 8) * x[g * group + k + 1];
      }
      acc += s * sc;
    }
    y[i] = acc;
  }
}

/* engine/weights.js:129-158 (_rawF16ToF32, the F16_LUT entries): IEEE half to float, exact */
static float f16_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000) << 16;
  int e = (h >> 10) & 0x1f;
  uint32_t f = h & 0x3ff, bits;
  if (e == 0) {
    if (f == 0) {
      bits = s;
    } else {
      e = 1;
      while ((f & 0x400) == 0) {
        f <<= 1;
        e -= 1;
      }
      f &= 0x3ff;
      bits = s | ((uint32_t)(e + 127 - 15) << 23) | (f << 13);
    }
  } else if (e == 31) {
    bits = s | 0x7f800000u | (f << 13);
  } else {
    bits = s | ((uint32_t)(e + 127 - 15) << 23) | (f << 13);
  }
  float v;
  memcpy(&v, &bits, 4);
  return v;
}
/* gemvBf16's conversion (engine/infer.js:66-77): the 16 bits become the top of an f32 */
static float bf16_to_f32(uint16_t h) {
  const uint32_t bits = (uint32_t)h << 16;
  float v;
  memcpy(&v, &bits, 4);
  return v;
}

/* gemvF32 / gemvF16 / gemvBf16 / gemvQ8 (engine/infer.js:10-86): a double accumulator (the JS `let s`)
   per row, products of f32 values in double, gemvF32's 8-way unrolled order, q8's row scale after the
   sum; each row stored as f32. */
static void gemv_dense(const otensor* w, const float* x, float* y) {
  const int n = w->cols;
  for (int i = 0; i < w->rows; i++) {
    double s = 0;
    if (w->storage == ST_F32) {
      const float* r = (const float*)w->data + (size_t)i * n;
      int k = 0;
      for (; k < n - 7; k += 8) {
        s += (double)r[k] * x[k];
        s += (double)r[k + 1] * x[k + 1];
        s += (double)r[k + 2] * x[k + 2];
        s += (double)r[k + 3] * x[k + 3];
        s += (double)r[k + 4] * x[k + 4];
        s += (double)r[k + 5] * x[k + 5];
        s += (double)r[k + 6] * x[k + 6];
        s += (double)r[k + 7] * x[k + 7];
      }
      for (; k < n; k++) s += (double)r[k] * x[k];
    } else if (w->storage == ST_F16) {
      const uint16_t* r = (const uint16_t*)w->data + (size_t)i * n;
      for (int k = 0; k < n; k++) s += (double)f16_to_f32(r[k]) * x[k];
    } else if (w->storage == ST_BF16) {
      const uint16_t* r = (const uint16_t*)w->data + (size_t)i * n;
      for (int k = 0; k < n; k++) s += (double)bf16_to_f32(r[k]) * x[k];
    } else { /* ST_Q8 */
      const int8_t* r = (const int8_t*)w->data + (size_t)i * n;
      for (int k = 0; k < n; k++) s += (double)r[k] * x[k];
      s = s * w->scale[i];
    }
    y[i] = (float)s;
  }
}

/* engine/infer.js:337-345 (gemv, dispatched on the tensor's storage) */
static void gemv_any(const oracle_model* m, const otensor* w, const float* x, float* y) {
  if (w->storage == ST_Q4)
    gemv_q4_pool(m->pool, w->rows, w->cols, w->data, w->scale, w->group, x, y);
  else
    gemv_dense(w, x, y);
}

/* engine/infer.js:118-132 — t independent GEMVs */
static void gemm_q4(const oracle_model* m, const otensor* w, int t, const float* x, float* y) {
  for (int i = 0; i < t; i++) gemv_any(m, w, x + (size_t)i * w->cols, y + (size_t)i * w->rows);
}

/* ------------------------------------------------------------------------------------------ */
/* elementwise ops                                                                            */
/* ------------------------------------------------------------------------------------------ */

/* engine/infer.js:134-143 */
static void rms_norm(const float* x, const float* w, float* out, int dim, int tokens) {
  for (int t = 0; t < tokens; t++) {
    const float* xo = x + (size_t)t * dim;
    float* oo = out + (size_t)t * dim;
    double ss = 0;
    for (int i = 0; i < dim; i++) ss += (double)xo[i] * xo[i];
    const double inv = 1 / sqrt(ss / dim + EPS);
    for (int i = 0; i < dim; i++) oo[i] = (float)((double)xo[i] * inv * w[i]);
  }
}

/* engine/infer.js:147-164 */
static void layer_norm(const float* x, const float* wb, float* out, int dim, int tokens) {
  for (int t = 0; t < tokens; t++) {
    const float* xo = x + (size_t)t * dim;
    float* oo = out + (size_t)t * dim;
    double mean = 0;
    for (int i = 0; i < dim; i++) mean += xo[i];
    mean /= dim;
    double v = 0;
    for (int i = 0; i < dim; i++) {
      const double del = xo[i] - mean;
      v += del * del;
    }
    const double inv = 1 / sqrt(v / dim + LN_EPS);
    for (int i = 0; i < dim; i++) oo[i] = (float)((xo[i] - mean) * inv * wb[i] + wb[dim + i]);
  }
}

/* engine/infer.js:166-171 */
static void gelu_new_inplace(float* a, int n) {
  for (int i = 0; i < n; i++) {
    const double v = a[i];
    a[i] = (float)(0.5 * v * (1 + tanh(0.7978845608028654 * (v + 0.044715 * v * v * v))));
  }
}

/* engine/infer.js:173-176 */
static void add_bias(float* y, const float* b, int n) {
  if (!b) return;
  for (int i = 0; i < n; i++) y[i] = (float)((double)y[i] + b[i]);
}

/* engine/infer.js:178-183 */
static void silu_mul(float* a, const float* b, int n) {
  for (int i = 0; i < n; i++) {
    const double v = a[i];
    a[i] = (float)((v / (1 + exp(-v))) * b[i]);
  }
}

/* engine/infer.js:185-206 */
static void build_rope(oracle_model* m) {
  const int hd = m->head_dim;
  int ropeDim = (int)floor(hd * m->c.rope_pct);
  ropeDim -= ropeDim % 2;
  const int half = ropeDim / 2;
  m->rope_dim = ropeDim;
  float* inv = (float*)malloc(sizeof(float) * (half > 0 ? half : 1));
  for (int i = 0; i < half; i++) inv[i] = (float)(1 / pow(m->c.rope_theta, (double)(2 * i) / ropeDim));
  const size_t n = (size_t)m->c.max_seq * (ropeDim > 0 ? ropeDim : 1);
  m->rope_cos = (float*)calloc(n, sizeof(float));
  m->rope_sin = (float*)calloc(n, sizeof(float));
  for (int t = 0; t < m->c.max_seq; t++) {
    for (int i = 0; i < half; i++) {
      const double freq = (double)t * inv[i];
      const double c = cos(freq), s = sin(freq);
      m->rope_cos[(size_t)t * ropeDim + i] = (float)c;
      m->rope_cos[(size_t)t * ropeDim + half + i] = (float)c;
      m->rope_sin[(size_t)t * ropeDim + i] = (float)s;
      m->rope_sin[(size_t)t * ropeDim + half + i] = (float)s;
    }
  }
  free(inv);
}

/* engine/infer.js:208-225 — qOrK laid out [nHeads][t][hd] */
static void apply_rope(const oracle_model* m, float* qk, int nHeads, int t, int offset) {
  const int ropeDim = m->rope_dim, half = ropeDim / 2, hd = m->head_dim;
  float rot[512];
  for (int h = 0; h < nHeads; h++) {
    for (int ti = 0; ti < t; ti++) {
      const int pos = offset + ti;
      float* base = qk + ((size_t)h * t + ti) * hd;
      const float* cs = m->rope_cos + (size_t)pos * ropeDim;
      const float* sn = m->rope_sin + (size_t)pos * ropeDim;
      for (int i = 0; i < half; i++) rot[i] = -base[half + i];
      for (int i = 0; i < half; i++) rot[half + i] = base[i];
      for (int i = 0; i < ropeDim; i++) base[i] = (float)((double)base[i] * cs[i] + (double)rot[i] * sn[i]);
    }
  }
}

/* engine/infer.js:227-238 */
static void softmax_inplace(float* x, int n) {
  double max = -INFINITY;
  for (int i = 0; i < n; i++)
    if (x[i] > max) max = x[i];
  double s = 0;
  for (int i = 0; i < n; i++) {
    const double e = exp(x[i] - max);
    x[i] = (float)e;
    s += e;
  }
  const double inv = 1 / s;
  for (int i = 0; i < n; i++) x[i] = (float)(x[i] * inv);
}

/* engine/infer.js:240-250 */
int oracle_argmax(const float* logits, int n) {
  int bi = 0;
  float bv = logits[0];
  for (int i = 1; i < n; i++)
    if (logits[i] > bv) {
      bv = logits[i];
      bi = i;
    }
  return bi;
}

/* engine/infer.js:252-287 (noRepeatNgram = 3, penalty = 1.15) */
int oracle_argmax_gpt2(const float* logits, int n, const int32_t* history, int n_past) {
  const double penalty = 1.15;
  int t1 = -1, t2 = -1;
  if (n_past >= 2) {
    t1 = history[n_past - 2];
    t2 = history[n_past - 1];
  }
  int bestIdx = 0;
  double bestVal = -INFINITY;
  const int recentWin = n_past - 32 > 0 ? n_past - 32 : 0;
  for (int i = 0; i < n; i++) {
    double v = logits[i];
    if (n_past >= 2) {
      for (int h = 0; h < n_past - 2; h++) {
        if (history[h] == t1 && history[h + 1] == t2 && history[h + 2] == i) {
          v = -1e9;
          break;
        }
      }
    }
    if (penalty > 1.0 && v > -1e8) {
      for (int h = recentWin; h < n_past; h++) {
        if (history[h] == i) {
          v = v > 0 ? v / penalty : v * penalty;
          break;
        }
      }
    }
    if (v > bestVal) {
      bestVal = v;
      bestIdx = i;
    }
  }
  return bestIdx;
}

/* ------------------------------------------------------------------------------------------ */
/* model                                                                                      */
/* ------------------------------------------------------------------------------------------ */

static const otensor* find(const oracle_model* m, const char* name) {
  for (int i = 0; i < m->n_tensors; i++)
    if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
  return NULL;
}

static const float* find_f32(const oracle_model* m, const char* name) {
  const otensor* t = find(m, name);
  return (t && t->storage == ST_F32) ? (const float*)t->data : NULL;
}

/* Create a model from a parsed PGW1 table.  Tensor data stays owned by the caller. */
oracle_model* oracle_create(const int* cfg_i, const double* cfg_d, int n_tensors, const char* const* names,
                            const int* storage, const int* rows, const int* cols, const int* group,
                            const void* const* data, const void* const* scale) {
  oracle_model* m = (oracle_model*)calloc(1, sizeof(oracle_model));
  m->c.arch = cfg_i[0];
  m->c.vocab = cfg_i[1];
  m->c.n_layers = cfg_i[2];
  m->c.d_model = cfg_i[3];
  m->c.n_heads = cfg_i[4];
  m->c.n_kv_heads = cfg_i[5];
  m->c.d_ff = cfg_i[6];
  m->c.max_seq = cfg_i[7];
  m->c.rope_theta = cfg_d[0];
  m->c.rope_pct = cfg_d[1];
  m->head_dim = m->c.d_model / m->c.n_heads;
  m->kv_dim = m->c.n_kv_heads * m->head_dim;
  m->rep = m->c.n_heads / m->c.n_kv_heads;
  m->threads = 1;
  m->n_tensors = n_tensors;
  m->tensors = (otensor*)calloc(n_tensors, sizeof(otensor));
  for (int i = 0; i < n_tensors; i++) {
    otensor* t = &m->tensors[i];
    strncpy(t->name, names[i], sizeof(t->name) - 1);
    t->storage = storage[i];
    t->rows = rows[i];
    t->cols = cols[i];
    t->group = group[i] ? group[i] : 32;
    t->data = (const uint8_t*)data[i];
    t->scale = (const float*)scale[i];
  }
  const int L = m->c.n_layers;
  m->qkv = calloc(L, sizeof(void*));
  m->proj = calloc(L, sizeof(void*));
  m->w1 = calloc(L, sizeof(void*));
  m->w3 = calloc(L, sizeof(void*));
  m->w2 = calloc(L, sizeof(void*));
  m->norm1 = calloc(L, sizeof(void*));
  m->norm2 = calloc(L, sizeof(void*));
  m->qkv_b = calloc(L, sizeof(void*));
  m->proj_b = calloc(L, sizeof(void*));
  m->fc_b = calloc(L, sizeof(void*));
  m->mproj_b = calloc(L, sizeof(void*));
  char nm[96];
  m->lm_head = find(m, "lm_head");
  const int gpt2 = m->c.arch == 1;
  for (int l = 0; l < L; l++) {
    snprintf(nm, sizeof nm, "blocks.%d.attn.qkv", l); m->qkv[l] = find(m, nm);
    snprintf(nm, sizeof nm, "blocks.%d.attn.proj", l); m->proj[l] = find(m, nm);
    if (gpt2) {
      snprintf(nm, sizeof nm, "blocks.%d.mlp.fc", l); m->w1[l] = find(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.mlp.proj", l); m->w2[l] = find(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.ln1", l); m->norm1[l] = find_f32(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.ln2", l); m->norm2[l] = find_f32(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.attn.qkv_bias", l); m->qkv_b[l] = find_f32(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.attn.proj_bias", l); m->proj_b[l] = find_f32(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.mlp.fc_bias", l); m->fc_b[l] = find_f32(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.mlp.proj_bias", l); m->mproj_b[l] = find_f32(m, nm);
    } else {
      snprintf(nm, sizeof nm, "blocks.%d.mlp.w1", l); m->w1[l] = find(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.mlp.w3", l); m->w3[l] = find(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.mlp.w2", l); m->w2[l] = find(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.norm1", l); m->norm1[l] = find_f32(m, nm);
      snprintf(nm, sizeof nm, "blocks.%d.norm2", l); m->norm2[l] = find_f32(m, nm);
    }
  }
  m->norm_f = find_f32(m, gpt2 ? "ln_f" : "norm_f");
  m->wpe = find_f32(m, "wpe");
  m->scale_factors = find_f32(m, "scale_factors");
  if (!gpt2) build_rope(m);
  const size_t kvn = (size_t)m->c.n_kv_heads * m->c.max_seq * m->head_dim;
  m->k_cache = calloc(L, sizeof(float*));
  m->v_cache = calloc(L, sizeof(float*));
  for (int l = 0; l < L; l++) {
    m->k_cache[l] = (float*)calloc(kvn, sizeof(float));
    m->v_cache[l] = (float*)calloc(kvn, sizeof(float));
  }
  m->cache_len = 0;
  return m;
}

/* Returns 0 when every tensor the forward needs is present. */
int oracle_check(const oracle_model* m) {
  if (!m->lm_head || !m->norm_f) return -1;
  for (int l = 0; l < m->c.n_layers; l++) {
    if (!m->qkv[l] || !m->proj[l] || !m->w1[l] || !m->w2[l] || !m->norm1[l] || !m->norm2[l]) return -2 - l;
    if (m->c.arch == 0 && !m->w3[l]) return -2 - l;
  }
  if (m->c.arch == 1 && !m->wpe) return -1000;
  return 0;
}

void oracle_set_threads(oracle_model* m, int threads) {
  m->threads = threads > 0 ? threads : 1;
  pool_destroy(m->pool);
  m->pool = m->threads > 1 ? pool_create(m->threads) : NULL;
}

void oracle_free(oracle_model* m) {
  if (!m) return;
  pool_destroy(m->pool);
  for (int l = 0; l < m->c.n_layers; l++) {
    free(m->k_cache[l]);
    free(m->v_cache[l]);
  }
  free(m->k_cache); free(m->v_cache);
  free(m->qkv); free(m->proj); free(m->w1); free(m->w3); free(m->w2);
  free(m->norm1); free(m->norm2); free(m->qkv_b); free(m->proj_b); free(m->fc_b); free(m->mproj_b);
  free(m->rope_cos); free(m->rope_sin);
  free(m->tensors);
  free(m);
}

/* engine/infer.js:348-358 */
void oracle_reset(oracle_model* m) {
  const size_t kvn = (size_t)m->c.n_kv_heads * m->c.max_seq * m->head_dim;
  for (int l = 0; l < m->c.n_layers; l++) {
    memset(m->k_cache[l], 0, kvn * sizeof(float));
    memset(m->v_cache[l], 0, kvn * sizeof(float));
  }
  m->cache_len = 0;
}

int oracle_cache_len(const oracle_model* m) { return m->cache_len; }
void oracle_set_cache_len(oracle_model* m, int n) { m->cache_len = n; }

/* engine/infer.js:395-420 (q8 and q4 branches) */
static void embed_row_quant(const oracle_model* m, int id, float* row) {
  const otensor* w = m->lm_head;
  const int n = m->c.d_model, group = w->group, packedRow = n / 2;
  int ng = n / group;
  if (w->storage == ST_Q8) {
    const float sc = w->scale[id];
    const int8_t* q = (const int8_t*)w->data + (size_t)id * n;
    for (int i = 0; i < n; i++) row[i] = (float)((double)q[i] * sc);
    ng = 0;
  }
  for (int g = 0; g < ng; g++) {
    const float sc = w->scale[(size_t)id * ng + g];
    const uint8_t* base = w->data + (size_t)id * packedRow + g * (group / 2);
    for (int k = 0; k < group; k += 2) {
      const int b = base[k / 2];
      row[g * group + k] = (float)((double)((b & 15) - 8) * sc);
      row[g * group + k + 1] = (float)((double)((b >> 4) - 8) * sc);
    }
  }
  if (m->c.arch == 1 && m->scale_factors)
    for (int i = 0; i < n; i++) row[i] = (float)((double)row[i] / m->scale_factors[i]);
}

/* engine/infer.js:360-393 */
static void embed(const oracle_model* m, const int32_t* ids, int t, float* out, int pos0) {
  const int d = m->c.d_model;
  const otensor* w = m->lm_head;
  for (int i = 0; i < t; i++) {
    float* row = out + (size_t)i * d;
    const size_t off = (size_t)ids[i] * d;
    if (w->storage == ST_F32) {
      memcpy(row, (const float*)w->data + off, (size_t)d * sizeof(float));
    } else if (w->storage == ST_F16) {
      for (int k = 0; k < d; k++) row[k] = f16_to_f32(((const uint16_t*)w->data)[off + k]);
    } else if (w->storage == ST_BF16) {
      for (int k = 0; k < d; k++) row[k] = bf16_to_f32(((const uint16_t*)w->data)[off + k]);
    } else {
      embed_row_quant(m, ids[i], row);
    }
  }
  if (m->c.arch == 1) {
    const int maxSeq = m->c.max_seq ? m->c.max_seq : 1024;
    for (int i = 0; i < t; i++) {
      const int safePos = pos0 + i < maxSeq - 1 ? pos0 + i : maxSeq - 1;
      for (int k = 0; k < d; k++)
        out[(size_t)i * d + k] = (float)((double)out[(size_t)i * d + k] + m->wpe[(size_t)safePos * d + k]);
    }
  }
}

typedef struct {
  float *x, *xn, *qkv, *q, *k, *v, *attn, *proj, *ff1, *ff3, *ff2, *scores, *yhead;
} scratch;

static void scratch_alloc(const oracle_model* m, int t, scratch* s) {
  const ocfg* c = &m->c;
  const int hd = m->head_dim;
  s->x = calloc((size_t)t * c->d_model, 4);
  s->xn = calloc((size_t)t * c->d_model, 4);
  s->qkv = calloc((size_t)t * (c->d_model + 2 * m->kv_dim), 4);
  s->q = calloc((size_t)c->n_heads * t * hd, 4);
  s->k = calloc((size_t)c->n_kv_heads * t * hd, 4);
  s->v = calloc((size_t)c->n_kv_heads * t * hd, 4);
  s->attn = calloc((size_t)t * c->d_model, 4);
  s->proj = calloc((size_t)t * c->d_model, 4);
  s->ff1 = calloc((size_t)t * c->d_ff, 4);
  s->ff3 = calloc((size_t)t * c->d_ff, 4);
  s->ff2 = calloc((size_t)t * c->d_model, 4);
  s->scores = calloc((size_t)c->max_seq, 4);
  s->yhead = calloc((size_t)hd, 4);
}

static void scratch_free(scratch* s) {
  free(s->x); free(s->xn); free(s->qkv); free(s->q); free(s->k); free(s->v); free(s->attn);
  free(s->proj); free(s->ff1); free(s->ff3); free(s->ff2); free(s->scores); free(s->yhead);
}

/* engine/infer.js:422-504 */
static const float* attention(oracle_model* m, scratch* s, int layer, const float* x, int t, int pastLen) {
  const ocfg* c = &m->c;
  const int nHeads = c->n_heads, nKv = c->n_kv_heads, dModel = c->d_model, hd = m->head_dim, kvDim = m->kv_dim;
  const int width = dModel + 2 * kvDim;
  gemm_q4(m, m->qkv[layer], t, x, s->qkv);
  if (c->arch == 1)
    for (int ti = 0; ti < t; ti++) add_bias(s->qkv + (size_t)ti * width, m->qkv_b[layer], width);
  for (int ti = 0; ti < t; ti++) {
    const float* src = s->qkv + (size_t)ti * width;
    for (int h = 0; h < nHeads; h++)
      for (int d = 0; d < hd; d++) s->q[((size_t)h * t + ti) * hd + d] = src[h * hd + d];
    for (int h = 0; h < nKv; h++)
      for (int d = 0; d < hd; d++) {
        s->k[((size_t)h * t + ti) * hd + d] = src[dModel + h * hd + d];
        s->v[((size_t)h * t + ti) * hd + d] = src[dModel + kvDim + h * hd + d];
      }
  }
  if (c->arch != 1) {
    apply_rope(m, s->q, nHeads, t, pastLen);
    apply_rope(m, s->k, nKv, t, pastLen);
  }
  float* kC = m->k_cache[layer];
  float* vC = m->v_cache[layer];
  const int seq = pastLen + t;
  for (int h = 0; h < nKv; h++)
    for (int ti = 0; ti < t; ti++) {
      const size_t dst = ((size_t)h * c->max_seq + pastLen + ti) * hd;
      const size_t src = ((size_t)h * t + ti) * hd;
      memcpy(kC + dst, s->k + src, hd * sizeof(float));
      memcpy(vC + dst, s->v + src, hd * sizeof(float));
    }
  const double scale = 1 / sqrt((double)hd);
  for (int h = 0; h < nHeads; h++) {
    const int kvh = h / m->rep;
    for (int qi = 0; qi < t; qi++) {
      const int qpos = pastLen + qi;
      const float* qv = s->q + ((size_t)h * t + qi) * hd;
      for (int kj = 0; kj < seq; kj++) {
        if (kj > qpos) {
          s->scores[kj] = -1e9f;
          continue;
        }
        const float* kr = kC + ((size_t)kvh * c->max_seq + kj) * hd;
        double dot = 0;
        for (int d = 0; d < hd; d++) dot += (double)qv[d] * kr[d];
        s->scores[kj] = (float)(dot * scale);
      }
      softmax_inplace(s->scores, seq);
      for (int d = 0; d < hd; d++) s->yhead[d] = 0;
      for (int kj = 0; kj < seq; kj++) {
        const float a = s->scores[kj];
        if (a == 0) continue;
        const float* vr = vC + ((size_t)kvh * c->max_seq + kj) * hd;
        for (int d = 0; d < hd; d++) s->yhead[d] = (float)((double)s->yhead[d] + (double)a * vr[d]);
      }
      memcpy(s->attn + ((size_t)qi * nHeads + h) * hd, s->yhead, hd * sizeof(float));
    }
  }
  gemm_q4(m, m->proj[layer], t, s->attn, s->proj);
  if (c->arch == 1)
    for (int ti = 0; ti < t; ti++) add_bias(s->proj + (size_t)ti * dModel, m->proj_b[layer], dModel);
  return s->proj;
}

/* engine/infer.js:506-527 */
static const float* ffn(oracle_model* m, scratch* s, int layer, const float* x, int t) {
  const ocfg* c = &m->c;
  const int n = t * c->d_ff;
  if (c->arch == 1) {
    gemm_q4(m, m->w1[layer], t, x, s->ff1);
    for (int ti = 0; ti < t; ti++) add_bias(s->ff1 + (size_t)ti * c->d_ff, m->fc_b[layer], c->d_ff);
    gelu_new_inplace(s->ff1, n);
    gemm_q4(m, m->w2[layer], t, s->ff1, s->ff2);
    for (int ti = 0; ti < t; ti++) add_bias(s->ff2 + (size_t)ti * c->d_model, m->mproj_b[layer], c->d_model);
    return s->ff2;
  }
  gemm_q4(m, m->w1[layer], t, x, s->ff1);
  gemm_q4(m, m->w3[layer], t, x, s->ff3);
  silu_mul(s->ff1, s->ff3, n);
  gemm_q4(m, m->w2[layer], t, s->ff1, s->ff2);
  return s->ff2;
}

/*
 * One forward over t tokens at positions pastLen..pastLen+t-1 (engine/infer.js:553-601; forwardPrompt
 * is pastLen = 0, forwardDecode is t = 1).  logits: [vocab] for the last row, or [t][vocab] when
 * logits_each (the verify forward of engine/webgpu.js:1248).  hidden (nullable): x after each layer,
 * [nLayers][t][d].  Returns 0 on success.
 */
int oracle_forward(oracle_model* m, const int32_t* ids, int t, int pastLen, int logits_each, float* logits,
                   float* hidden) {
  const ocfg* c = &m->c;
  const int d = c->d_model;
  if (t <= 0 || pastLen < 0 || pastLen + t > c->max_seq) return -1;
  for (int i = 0; i < t; i++)
    if (ids[i] < 0 || ids[i] >= c->vocab) return -2;
  scratch s;
  scratch_alloc(m, t, &s);
  embed(m, ids, t, s.x, pastLen);
  for (int li = 0; li < c->n_layers; li++) {
    if (c->arch == 1) layer_norm(s.x, m->norm1[li], s.xn, d, t);
    else rms_norm(s.x, m->norm1[li], s.xn, d, t);
    const float* att = attention(m, &s, li, s.xn, t, pastLen);
    for (int i = 0; i < t * d; i++) s.x[i] = (float)((double)s.x[i] + att[i]);
    if (c->arch == 1) layer_norm(s.x, m->norm2[li], s.xn, d, t);
    else rms_norm(s.x, m->norm2[li], s.xn, d, t);
    const float* ff = ffn(m, &s, li, s.xn, t);
    for (int i = 0; i < t * d; i++) s.x[i] = (float)((double)s.x[i] + ff[i]);
    if (hidden) memcpy(hidden + (size_t)li * t * d, s.x, (size_t)t * d * sizeof(float));
  }
  m->cache_len = pastLen + t;
  if (c->arch == 1) layer_norm(s.x, m->norm_f, s.xn, d, t);
  else rms_norm(s.x, m->norm_f, s.xn, d, t);
  const otensor* lm = m->lm_head;
  if (logits_each) {
    for (int i = 0; i < t; i++) gemv_any(m, lm, s.xn + (size_t)i * d, logits + (size_t)i * c->vocab);
  } else {
    gemv_any(m, lm, s.xn + (size_t)(t - 1) * d, logits);
  }
  scratch_free(&s);
  return 0;
}

enum { STOP_EOS = 0, STOP_MAX_NEW = 1, STOP_CONTEXT = 2 };

/*
 * engine/infer.js:603-646.  ids are used as given (the caller applies the prompt truncation of
 * infer.js:604-608).  out_ids has room for max_new ids.  step_logits (nullable): [max_new][vocab]
 * logits that produced each generated id.  Returns the number of generated ids, negative on error.
 */
int oracle_generate(oracle_model* m, const int32_t* ids, int n, int max_new, int32_t eos, int32_t* out_ids,
                    int* stop_reason, float* step_logits) {
  const ocfg* c = &m->c;
  const int V = c->vocab;
  float* logits = (float*)malloc(sizeof(float) * V);
  oracle_reset(m);
  int rc = oracle_forward(m, ids, n, 0, 0, logits, NULL);
  if (rc) {
    free(logits);
    return rc;
  }
  int nout = 0;
  int32_t next = c->arch == 1 ? oracle_argmax_gpt2(logits, V, out_ids, 0) : oracle_argmax(logits, V);
  if (step_logits) memcpy(step_logits, logits, sizeof(float) * V);
  out_ids[nout++] = next;
  *stop_reason = STOP_MAX_NEW;
  if (next == eos) {
    *stop_reason = STOP_EOS;
    free(logits);
    return nout;
  }
  for (int i = 1; i < max_new; i++) {
    if (n + nout >= c->max_seq) break;
    rc = oracle_forward(m, &next, 1, m->cache_len, 0, logits, NULL);
    if (rc) {
      free(logits);
      return rc;
    }
    next = c->arch == 1 ? oracle_argmax_gpt2(logits, V, out_ids, nout) : oracle_argmax(logits, V);
    if (step_logits) memcpy(step_logits + (size_t)nout * V, logits, sizeof(float) * V);
    out_ids[nout++] = next;
    if (next == eos) {
      *stop_reason = STOP_EOS;
      break;
    }
  }
  free(logits);
  return nout;
}

/* engine/webgpu.js:846-865 — returns the draft length, draft written to out (room for k ids) */
int oracle_lookup_draft(const int32_t* seq, int len, int k, int n, int32_t* out) {
  if (len < n + 1) return 0;
  const int32_t* suf = seq + len - n;
  const int limit = len - n;
  for (int i = limit - 1; i >= 0; i--) {
    int ok = 1;
    for (int j = 0; j < n; j++)
      if (seq[i + j] != suf[j]) {
        ok = 0;
        break;
      }
    if (ok) {
      int d = 0;
      for (int t = 0; t < k && i + n + t < len; t++) out[d++] = seq[i + n + t];
      return d;
    }
  }
  return 0;
}

/*
 * engine/webgpu.js:1164-1282, fused path with prompt-lookup speculation (llama arch).  Prefill of the
 * whole prompt, then per iteration: draft = lookupDraft(prompt + accepted, spec_k, ngram); one verify
 * forward over [last, ...draft] at pos = cacheLen with an argmax per row; accept r[0], then r[k+1]
 * while r[k] == draft[k].  The draft is cut so that every verify row stays inside the KV cache
 * (pos + len(draft) <= maxSeq - 1); the reference instead clamps KV row indices at maxSeq - 1
 * (engine/webgpu.js:457-468).  stats: [specHits, specTries, verify_forwards].  draft_log (nullable,
 * room for max_new * (spec_k + 2) ints): per iteration [len, draft..., n_accepted].
 */
int oracle_generate_spec(oracle_model* m, const int32_t* ids, int n, int max_new, int32_t eos, int spec_k,
                         int ngram, int32_t* out_ids, int* stop_reason, int* stats, int32_t* draft_log) {
  const ocfg* c = &m->c;
  const int V = c->vocab, maxSeq = c->max_seq;
  if (spec_k < 0 || spec_k > 64 || n <= 0) return -1;
  float* logits = (float*)malloc(sizeof(float) * V * (size_t)(spec_k + 1));
  int32_t* seq = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n + max_new + 1));
  int32_t draft[65], run[66], r[66];
  int specHits = 0, specTries = 0, forwards = 0, logpos = 0;
  oracle_reset(m);
  int rc = oracle_forward(m, ids, n, 0, 0, logits, NULL);
  if (rc) {
    free(logits);
    free(seq);
    return rc;
  }
  memcpy(seq, ids, sizeof(int32_t) * n);
  int seqLen = n, nacc = 0;
  out_ids[nacc++] = oracle_argmax(logits, V);
  seq[seqLen++] = out_ids[0];
  m->cache_len = n < maxSeq - 1 ? n : maxSeq - 1;
  *stop_reason = STOP_MAX_NEW;
  if (out_ids[0] == eos) {
    *stop_reason = STOP_EOS;
    goto done;
  }
  while (nacc < max_new) {
    if (m->cache_len >= maxSeq - 1) break;
    const int32_t x = out_ids[nacc - 1];
    const int pos = m->cache_len;
    int dl = oracle_lookup_draft(seq, seqLen, spec_k, ngram, draft);
    if (pos + dl > maxSeq - 1) dl = maxSeq - 1 - pos;
    specTries++;
    run[0] = x;
    for (int i = 0; i < dl; i++) run[1 + i] = draft[i];
    const int logitsEach = dl > 0;
    rc = oracle_forward(m, run, 1 + dl, pos, logitsEach, logits, NULL);
    forwards++;
    if (rc) {
      free(logits);
      free(seq);
      return rc;
    }
    for (int i = 0; i < 1 + dl; i++) r[i] = oracle_argmax(logits + (size_t)(logitsEach ? i : 0) * V, V);
    if (draft_log) {
      draft_log[logpos++] = dl;
      for (int i = 0; i < dl; i++) draft_log[logpos++] = draft[i];
    }
    int accepted_here = 0;
    out_ids[nacc++] = r[0];
    seq[seqLen++] = r[0];
    m->cache_len = pos + 1;
    if (r[0] != eos && dl && logitsEach) {
      for (int k = 0; k < dl; k++) {
        if (r[k] != draft[k]) break;
        if (nacc >= max_new) break;
        const int32_t nxt = r[k + 1];
        specHits++;
        accepted_here++;
        out_ids[nacc++] = nxt;
        seq[seqLen++] = nxt;
        m->cache_len = pos + 2 + k;
        if (nxt == eos) break;
      }
    }
    if (draft_log) draft_log[logpos++] = accepted_here;
    if (out_ids[nacc - 1] == eos) break;
  }
  if (out_ids[nacc - 1] == eos) *stop_reason = STOP_EOS;
done:
  if (stats) {
    stats[0] = specHits;
    stats[1] = specTries;
    stats[2] = forwards;
  }
  free(logits);
  free(seq);
  return nacc;
}
