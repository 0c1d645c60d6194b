// Allocation-free AdamW entry point (C ABI).
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
//  * The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; that set-up call
//    should happen before any stream capture begins.
//  * Every call shares the one array and it keeps the last call's contents.  Each call
//    writes every table entry it reads, so nothing in the array has to start at zero.
//    Two calls whose work overlaps on the GPU (for example on two streams) race on the
//    table: serialize them on one stream.
//  * No cudaMalloc, cudaFree or allocating library routine is called.  The table is
//    staged in a host-side static buffer and copied with cudaMemcpyAsync on the
//    caller's stream (from pageable memory, which the runtime stages before returning,
//    so the host buffer may be rewritten by the next call).
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace {

constexpr int kNoallocMaxTensors = 1024;
constexpr int kNoallocMaxDevices = 64;
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

// Host-side staging of the table (host memory; no device allocation involved).
static NoallocAdamEntry g_host_table[kNoallocMaxTensors];
static NoallocAdamEntry* g_table_dev_ptr[kNoallocMaxDevices] = {nullptr};
static char g_last_error[256] = "";

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

}  // namespace

extern "C" {

enum {
  TFB_NOALLOC_OK = 0,
  TFB_NOALLOC_TOO_MANY_TENSORS = 1,
  TFB_NOALLOC_BAD_ARGUMENT = 2,
  TFB_NOALLOC_CUDA_ERROR = 3,
};

// Largest tensor count one call accepts.
__attribute__((visibility("default"))) int tfb_adamw_noalloc_max_tensors(void) { return kNoallocMaxTensors; }

// Text of the last error reported by tfb_adamw_multi_noalloc (empty after success).
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
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) {
    set_error("tfb_adamw_multi_noalloc: no usable current CUDA device");
    return TFB_NOALLOC_CUDA_ERROR;
  }
  if (g_table_dev_ptr[dev] == nullptr) {
    // Once per device, with that device current: the array's device address.
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_adamw_table);
    if (e != cudaSuccess || ptr == nullptr) {
      set_error("tfb_adamw_multi_noalloc: cudaGetSymbolAddress of the static table failed");
      return TFB_NOALLOC_CUDA_ERROR;
    }
    g_table_dev_ptr[dev] = static_cast<NoallocAdamEntry*>(ptr);
  }
  long long chunks = 0;
  for (int i = 0; i < n_tensors; ++i) {
    if (numels[i] < 1 || !params[i] || !grads[i] || !exp_avgs[i] || !exp_avg_sqs[i]) {
      set_error("tfb_adamw_multi_noalloc: empty tensor or null pointer in the table");
      return TFB_NOALLOC_BAD_ARGUMENT;
    }
    g_host_table[i].p = params[i];
    g_host_table[i].g = grads[i];
    g_host_table[i].m = exp_avgs[i];
    g_host_table[i].v = exp_avg_sqs[i];
    g_host_table[i].n = numels[i];
    g_host_table[i].chunk0 = chunks;
    g_host_table[i].bc1 = bias1[i];
    g_host_table[i].bc2 = bias2[i];
    chunks += (numels[i] + kNoallocChunk - 1) / kNoallocChunk;
  }
  if (chunks > 0x7fffffffLL) {
    set_error("tfb_adamw_multi_noalloc: too many elements for one launch");
    return TFB_NOALLOC_BAD_ARGUMENT;
  }
  cudaError_t e = cudaMemcpyAsync(g_table_dev_ptr[dev], g_host_table, sizeof(NoallocAdamEntry) * n_tensors,
                                  cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) {
    set_error("tfb_adamw_multi_noalloc: table copy failed");
    return TFB_NOALLOC_CUDA_ERROR;
  }
  adamw_noalloc_kernel<<<(unsigned)chunks, 256, 0, stream>>>(g_table_dev_ptr[dev], n_tensors, lr_dev,
                                                             (float)(1.0 - beta1), (float)(1.0 - beta2),
                                                             eps, weight_decay, cautious);
  e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("tfb_adamw_multi_noalloc: kernel launch failed");
    return TFB_NOALLOC_CUDA_ERROR;
  }
  return TFB_NOALLOC_OK;
}

}  // extern "C"
