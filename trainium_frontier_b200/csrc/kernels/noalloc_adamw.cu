// Allocation-free AdamW entry point (C ABI); declarations in noalloc_adamw.h.
//
// This file has no counterpart in the reference implementation; it is an addition
// for callers of this library that must not allocate device memory.
//
// Who needs it.  The regular entry point (`adamw_multi` in optim_kernels.cu) builds
// its tensor table in device memory that it allocates on every call.  Some callers
// cannot allow that: a host runtime that reserves all of the GPU's memory for its own
// fixed arena at start-up and forbids any later cudaMalloc; a latency-critical loop in
// which a cudaMalloc / cudaFree could synchronize the whole device and stall other
// streams; a plain C caller that has no PyTorch caching allocator to borrow from.
// `tfb_adamw_multi_noalloc` serves them: the caller passes its own parameter,
// gradient and moment buffers (inputs and outputs), and the only extra device memory
// the kernel touches -- the tensor table -- lives in the file-scope array
// `g_noalloc_adamw_table` below, compiled into the library.
//
// Limits and rules.
//  * At most kNoallocMaxTensors (1024) tensors per call; larger calls are rejected
//    with TFB_NOALLOC_TOO_MANY_TENSORS and nothing is launched.  The array costs
//    1024 * 64 B = 64 KiB of device memory on every GPU that loads the library, held
//    until the process exits.
//  * Every call looks up the array's device address with cudaGetSymbolAddress, with
//    the caller's device current (a lookup allocates nothing), so the address is
//    never stale, e.g. after a cudaDeviceReset.
//  * Every call shares the one array and it keeps the last call's contents.  Each call
//    writes every table entry it reads, so nothing in the array has to start at zero.
//    Two calls whose work overlaps on the GPU (for example on two streams) race on the
//    table: serialize them on one stream.
//  * Host threads may call concurrently: a process-wide lock covers the host staging
//    buffer, the table copy and the launch, and the error message is kept per thread.  Their GPU
//    work still shares the one table, so the rule above applies across threads too.
//  * The table is copied with cudaMemcpyAsync on the caller's stream from a pageable
//    host buffer.  The runtime stages that copy before returning, so the buffer can be
//    reused at once, but it may first wait for the stream's earlier work: a call can
//    block the host until the stream drains.  For the same reason a call made while
//    the stream is being captured into a CUDA graph is not supported.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include "noalloc_adamw.h"

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

namespace {

constexpr int kNoallocMaxTensors = 1024;
constexpr int kNoallocChunk = 8192;

struct __align__(64) NoallocAdamEntry {
  float* p;
  const float* g;
  float* m;
  float* v;
  long long n;
  long long chunk0;
  float bc1, bc2;
};

// The scratch: the tensor table every call of the entry point writes and reads.
static __device__ __align__(256) NoallocAdamEntry g_noalloc_adamw_table[kNoallocMaxTensors];

// Host-side staging of the table (host memory; no device allocation involved), guarded
// by g_stage_lock from the first write until the copy has been staged by the runtime.
static NoallocAdamEntry g_host_table[kNoallocMaxTensors];
static std::mutex g_stage_lock;
static thread_local char g_last_error[256] = "";

__device__ __forceinline__ float lerp_torch(float a, float b, float w) {
  return (fabsf(w) < 0.5f) ? a + w * (b - a) : b - (b - a) * (1.f - w);
}

// Same arithmetic as the regular AdamW kernel; the table comes from `tab`, the device
// address of g_noalloc_adamw_table.
__global__ void adamw_noalloc_kernel(const NoallocAdamEntry* __restrict__ tab, int ntab,
                                     const float* __restrict__ lr_ptr, float one_m_b1, float one_m_b2, float eps,
                                     float wd, int cautious) {
  const long long chunk = blockIdx.x;
  int lo = 0, hi = ntab - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab[mid].chunk0 <= chunk) lo = mid;
    else hi = mid - 1;
  }
  const NoallocAdamEntry e = tab[lo];
  const long long start = (chunk - e.chunk0) * kNoallocChunk;
  const long long end = start + kNoallocChunk < e.n ? start + kNoallocChunk : e.n;
  const float lr = *lr_ptr;
  const float decay = 1.f - lr * wd;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = e.g[i];
    const float m = lerp_torch(e.m[i], g, one_m_b1);
    const float v = lerp_torch(e.v[i], g * g, one_m_b2);
    e.m[i] = m;
    e.v[i] = v;
    const float d = sqrtf(v / e.bc2) + eps;
    const float u = (m / e.bc1) / d;
    float p = e.p[i];
    if (wd != 0.f) {
      if (cautious) p = p * (1.f - lr * wd * ((u * p) > 0.f ? 1.f : 0.f));
      else p = p * decay;
    }
    e.p[i] = p - u * lr;
  }
}

void set_error(const char* msg) {
  strncpy(g_last_error, msg, sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = '\0';
}

void set_cuda_error(const char* what, cudaError_t e) {
  snprintf(g_last_error, sizeof(g_last_error), "tfb_adamw_multi_noalloc: %s: %s (%s)", what, cudaGetErrorName(e),
           cudaGetErrorString(e));
}

}  // namespace

extern "C" {

// Largest tensor count one call accepts.
__attribute__((visibility("default"))) int tfb_adamw_noalloc_max_tensors(void) { return kNoallocMaxTensors; }

// Text of the calling thread's last error from tfb_adamw_multi_noalloc (empty after success).
__attribute__((visibility("default"))) const char* tfb_adamw_noalloc_last_error(void) { return g_last_error; }

// One AdamW step over `n_tensors` fp32 tensors, in place, on `stream`.
//   params, grads, exp_avgs, exp_avg_sqs : host arrays of device pointers (n_tensors each)
//   numels                               : host array of element counts
//   bias1, bias2                         : host arrays, 1 - beta^step per tensor
//   lr_dev                               : device pointer to the fp32 learning rate
// Arithmetic (per element, in this order): m = lerp(m, g, 1-beta1);
//   v = lerp(v, g*g, 1-beta2); u = (m / bias1) / (sqrt(v / bias2) + eps);
//   p *= 1 - lr*wd (cautious: only where u*p > 0); p -= u * lr.
// Returns TFB_NOALLOC_OK or an error code (see tfb_adamw_noalloc_last_error()).
__attribute__((visibility("default"))) int tfb_adamw_multi_noalloc(
    float* const* params, const float* const* grads, float* const* exp_avgs, float* const* exp_avg_sqs,
    const long long* numels, const float* bias1, const float* bias2, int n_tensors, const float* lr_dev,
    double beta1, double beta2, float eps, float weight_decay, int cautious, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (n_tensors < 1 || !params || !grads || !exp_avgs || !exp_avg_sqs || !numels || !bias1 || !bias2 || !lr_dev) {
    set_error("tfb_adamw_multi_noalloc: missing argument or n_tensors < 1");
    return TFB_NOALLOC_BAD_ARGUMENT;
  }
  if (n_tensors > kNoallocMaxTensors) {
    set_error("tfb_adamw_multi_noalloc: n_tensors exceeds the static table (1024 tensors); split the call");
    return TFB_NOALLOC_TOO_MANY_TENSORS;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error("cudaGetDevice", e);
    return TFB_NOALLOC_CUDA_ERROR;
  }
  // The array's device address on the current device (looked up on every call).
  void* table_dev = nullptr;
  e = cudaGetSymbolAddress(&table_dev, g_noalloc_adamw_table);
  if (e != cudaSuccess || table_dev == nullptr) {
    set_cuda_error("cudaGetSymbolAddress of the static table", e);
    return TFB_NOALLOC_CUDA_ERROR;
  }
  long long chunks = 0;
  for (int i = 0; i < n_tensors; ++i) {
    if (numels[i] < 1 || !params[i] || !grads[i] || !exp_avgs[i] || !exp_avg_sqs[i]) {
      set_error("tfb_adamw_multi_noalloc: empty tensor or null pointer in the table");
      return TFB_NOALLOC_BAD_ARGUMENT;
    }
    chunks += (numels[i] + kNoallocChunk - 1) / kNoallocChunk;
  }
  if (chunks > 0x7fffffffLL) {
    set_error("tfb_adamw_multi_noalloc: too many elements for one launch");
    return TFB_NOALLOC_BAD_ARGUMENT;
  }
  {
    std::lock_guard<std::mutex> lock(g_stage_lock);
    long long c = 0;
    for (int i = 0; i < n_tensors; ++i) {
      g_host_table[i].p = params[i];
      g_host_table[i].g = grads[i];
      g_host_table[i].m = exp_avgs[i];
      g_host_table[i].v = exp_avg_sqs[i];
      g_host_table[i].n = numels[i];
      g_host_table[i].chunk0 = c;
      g_host_table[i].bc1 = bias1[i];
      g_host_table[i].bc2 = bias2[i];
      c += (numels[i] + kNoallocChunk - 1) / kNoallocChunk;
    }
    // From pageable memory: staged by the runtime before this returns.  The launch stays
    // under the lock too, so on one stream every copy is followed by its own kernel.
    e = cudaMemcpyAsync(table_dev, g_host_table, sizeof(NoallocAdamEntry) * n_tensors, cudaMemcpyHostToDevice,
                        stream);
    if (e != cudaSuccess) {
      set_cuda_error("table copy (cudaMemcpyAsync)", e);
      return TFB_NOALLOC_CUDA_ERROR;
    }
    adamw_noalloc_kernel<<<(unsigned)chunks, 256, 0, stream>>>(static_cast<const NoallocAdamEntry*>(table_dev),
                                                               n_tensors, lr_dev, (float)(1.0 - beta1),
                                                               (float)(1.0 - beta2), eps, weight_decay, cautious);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    set_cuda_error("kernel launch", e);
    return TFB_NOALLOC_CUDA_ERROR;
  }
  return TFB_NOALLOC_OK;
}

}  // extern "C"
