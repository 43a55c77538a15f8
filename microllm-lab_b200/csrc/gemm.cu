// Q4 GEMM over T activation rows on the tensor cores (mllm_gemm_q4): the batched / skinny form of
// gemvQ4 (engine/infer.js:88-116) used for prefill, verify and multi-sequence decode.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <vector>

#include "../../include/mllm.h"
#include "q4mma.cuh"

namespace mllm {
void set_global_error(const char* msg);  // engine.cu: message for mllm_last_error(NULL)
}

namespace mllm {

// f32 [T][K] -> fp16 hi, lo [T][K]
__global__ void split_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    __half h, l;
    split_hi_lo(x[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}

template <int TBW>
__global__ void __launch_bounds__(kGemmThreads) gemm_store_kernel(const uint8_t* W, const float* S, const __half* xh,
                                                                  const __half* xl, float* Y, int R, int K, int T) {
  extern __shared__ __align__(16) unsigned char smem[];
  q4_gemm_tile<TBW>(W, S, xh, xl, K, R, K, T, blockIdx.x * kGemmRows, blockIdx.y * 8 * TBW, smem,
                    [&](int r, int t, float v) { Y[(size_t)t * R + r] = v; });
}

cudaError_t launch_gemm_store(const uint8_t* W, const float* S, const __half* xh, const __half* xl, float* Y, int R,
                              int K, int T, cudaStream_t st) {
  const dim3 grid((R + kGemmRows - 1) / kGemmRows, 1);
  if (T <= 16) {
    constexpr size_t sm = q4_gemm_smem_bytes<2>();
    gemm_store_kernel<2><<<dim3(grid.x, (T + 15) / 16), kGemmThreads, sm, st>>>(W, S, xh, xl, Y, R, K, T);
  } else {
    constexpr size_t sm = q4_gemm_smem_bytes<8>();
    gemm_store_kernel<8><<<dim3(grid.x, (T + 63) / 64), kGemmThreads, sm, st>>>(W, S, xh, xl, Y, R, K, T);
  }
  return cudaGetLastError();
}

// gemm_tc5.cu: the tcgen05 GEMM and the tiled activation halves it reads
cudaError_t launch_gemm_tc5(const uint8_t* W, const float* S, const __half* xh, const __half* xl, float* Y, int R,
                            int K, int T, cudaStream_t st);
cudaError_t launch_split_tiled(const float* x, __half* hi, __half* lo, int T, int K, cudaStream_t st);
size_t tc5_tiled_halves(int T, int K);

// Up to 16 activation rows the mma.sync tile (one 16-token pass, no tensor-memory set-up) is the faster
// of the two; from 17 rows on the tcgen05 GEMM is.
bool use_tc5(int n_act) { return n_act > 16; }

cudaError_t launch_split(const float* x, __half* hi, __half* lo, size_t n, cudaStream_t st) {
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  split_kernel<<<blocks, 256, 0, st>>>(x, hi, lo, n);
  return cudaGetLastError();
}

namespace {
// Per-device workspace for the fp16 halves of the activations.  It grows on demand; a superseded
// buffer is kept (not freed) until exit, because work already enqueued by an earlier call on some
// stream may still read it.  Growth is geometric, so few buffers are ever retired.
struct Workspace {
  std::mutex mu;
  std::vector<void*> ptr;
  std::vector<size_t> cap;
  std::vector<void*> retired;
};
Workspace g_ws;

// Called with g_ws.mu held.
int workspace_locked(size_t bytes, __half** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MLLM_ERR_CUDA;
  if ((int)g_ws.ptr.size() <= dev) {
    g_ws.ptr.resize(dev + 1, nullptr);
    g_ws.cap.resize(dev + 1, 0);
  }
  if (g_ws.cap[dev] < bytes) {
    const size_t want = std::max(bytes, 2 * g_ws.cap[dev]);
    void* p = nullptr;
    if (cudaMalloc(&p, want) != cudaSuccess) return MLLM_ERR_OOM;
    if (g_ws.ptr[dev]) g_ws.retired.push_back(g_ws.ptr[dev]);
    g_ws.ptr[dev] = p;
    g_ws.cap[dev] = want;
  }
  *out = (__half*)g_ws.ptr[dev];
  return MLLM_OK;
}
}  // namespace

}  // namespace mllm

extern "C" int mllm_gemm_q4(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y, int rows,
                            int cols, int n_act, void* stream) {
  using namespace mllm;
  if (!d_packed || !d_scales || !d_x || !d_y || rows <= 0 || cols <= 0 || cols % 32 || n_act <= 0) return MLLM_ERR_ARG;
  if (((uintptr_t)d_packed & 15) || ((uintptr_t)d_scales & 3) || ((uintptr_t)d_x & 3)) return MLLM_ERR_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const bool tc5 = use_tc5(n_act);
  const size_t n = tc5 ? tc5_tiled_halves(n_act, cols) : (size_t)n_act * cols;
  // The lock is held until both kernels are enqueued, so no other call can replace the workspace in
  // between.  Calls whose kernels overlap on the GPU (different streams or threads) still share the
  // workspace and must be serialised by the caller.
  std::lock_guard<std::mutex> lk(g_ws.mu);
  __half* ws = nullptr;
  int rc = workspace_locked(2 * n * sizeof(__half) + 256, &ws);
  if (rc) return rc;
  __half* hi = ws;
  __half* lo = ws + ((n + 127) / 128) * 128;
  if (tc5) {
    if (launch_split_tiled(d_x, hi, lo, n_act, cols, st) != cudaSuccess) return MLLM_ERR_CUDA;
    if (launch_gemm_tc5(d_packed, d_scales, hi, lo, d_y, rows, cols, n_act, st) != cudaSuccess) return MLLM_ERR_CUDA;
  } else {
    if (launch_split(d_x, hi, lo, n, st) != cudaSuccess) return MLLM_ERR_CUDA;
    if (launch_gemm_store(d_packed, d_scales, hi, lo, d_y, rows, cols, n_act, st) != cudaSuccess) return MLLM_ERR_CUDA;
  }
  return MLLM_OK;
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot call cudaMalloc: a host runtime that hands all
// device memory to its own pool up front (an extra allocation would fail or break its budget), or a
// latency-sensitive thread that cannot afford cudaMalloc's implicit device synchronisation.  This
// entry point keeps its scratch — the fp16 hi and lo halves of the activations — in a fixed array
// compiled into the library, so it allocates nothing at any call.
// ---------------------------------------------------------------------------------------------
namespace mllm {
namespace {

constexpr size_t kNoAllocMaxValues = size_t(1) << 20;  // n_act * cols <= 1,048,576 activation values
// hi halves in [0, max), lo halves in [max, 2 max): 4 MiB, held by every device that loads the library
static __device__ __align__(256) __half g_noalloc_scratch[2 * kNoAllocMaxValues];

std::mutex g_noalloc_mu;
std::vector<__half*> g_noalloc_addr;  // device address of g_noalloc_scratch, per device

// On the first call on a device (that device current) the array's device address is looked up;
// host code must never pass the symbol itself to a kernel.
int noalloc_scratch(__half** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    set_global_error("mllm_gemm_q4_noalloc: no current CUDA device");
    return MLLM_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if ((int)g_noalloc_addr.size() <= dev) g_noalloc_addr.resize(dev + 1, nullptr);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_global_error("mllm_gemm_q4_noalloc: cudaGetSymbolAddress failed for the scratch array");
      return MLLM_ERR_CUDA;
    }
    g_noalloc_addr[dev] = (__half*)p;
  }
  *out = g_noalloc_addr[dev];
  return MLLM_OK;
}

}  // namespace
}  // namespace mllm

extern "C" int mllm_gemm_q4_noalloc(const uint8_t* d_packed, const float* d_scales, const float* d_x, float* d_y,
                                    int rows, int cols, int n_act, void* stream) {
  using namespace mllm;
  if (!d_packed || !d_scales || !d_x || !d_y || rows <= 0 || cols <= 0 || cols % 32 || n_act <= 0) {
    set_global_error("mllm_gemm_q4_noalloc: null pointer, non-positive size or cols not a multiple of 32");
    return MLLM_ERR_ARG;
  }
  if (((uintptr_t)d_packed & 15) || ((uintptr_t)d_scales & 3) || ((uintptr_t)d_x & 3)) {
    set_global_error("mllm_gemm_q4_noalloc: misaligned device pointer");
    return MLLM_ERR_ARG;
  }
  const size_t n = (size_t)n_act * cols;
  if (n > kNoAllocMaxValues) {
    set_global_error("mllm_gemm_q4_noalloc: n_act * cols exceeds the fixed scratch of 1,048,576 values");
    return MLLM_ERR_ARG;
  }
  __half* base = nullptr;
  const int rc = noalloc_scratch(&base);
  if (rc) return rc;
  // Every element the GEMM reads is written by the split kernel of the same call, so nothing has
  // to start at zero; concurrent calls on overlapping streams share the array and race.
  __half* hi = base;
  __half* lo = base + kNoAllocMaxValues;
  cudaStream_t st = (cudaStream_t)stream;
  if (use_tc5(n_act) && tc5_tiled_halves(n_act, cols) <= kNoAllocMaxValues) {
    if (launch_split_tiled(d_x, hi, lo, n_act, cols, st) != cudaSuccess) return MLLM_ERR_CUDA;
    if (launch_gemm_tc5(d_packed, d_scales, hi, lo, d_y, rows, cols, n_act, st) != cudaSuccess) return MLLM_ERR_CUDA;
    return MLLM_OK;
  }
  // the tiled halves pad n_act to a multiple of 8 and would not fit: row-major halves instead
  if (launch_split(d_x, hi, lo, n, st) != cudaSuccess) return MLLM_ERR_CUDA;
  if (launch_gemm_store(d_packed, d_scales, hi, lo, d_y, rows, cols, n_act, st) != cudaSuccess) return MLLM_ERR_CUDA;
  return MLLM_OK;
}
