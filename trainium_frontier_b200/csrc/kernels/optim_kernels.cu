// Optimizer kernels.
//
// adamw_multi: one launch updates every tensor of an AdamW group (multi-tensor apply).
// Each CTA walks a chunk of one tensor; the tensor table (param / grad / exp_avg /
// exp_avg_sq pointers, sizes, per-tensor bias corrections) lives in device memory.
// Arithmetic order is the reference's foreach chain (train.py:3961-4021):
//   m = lerp(m, g, 1-b1); v = lerp(v, g*g, 1-b2); d = sqrt(v / bc2) + eps;
//   u = (m / bc1) / d; [p *= 1 - lr*wd (or cautious: only where u*p > 0)]; p -= u*lr
// with torch's lerp formula (a + w (b - a) for w < 0.5, else b - (b - a)(1 - w)).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

struct AdamEntry {
  float* p;
  const float* g;
  float* m;
  float* v;
  long long n;
  float bc1, bc2;
  long long chunk0;  // first chunk index of this tensor
};

__device__ __forceinline__ float torch_lerp(float a, float b, float w) {
  return (fabsf(w) < 0.5f) ? a + w * (b - a) : b - (b - a) * (1.f - w);
}

constexpr int kAdamChunk = 8192;

__global__ void adamw_multi_kernel(const AdamEntry* __restrict__ tab, int ntab, const float* __restrict__ lr_ptr,
                                   float one_m_b1, float one_m_b2, float eps, float wd, int cautious) {
  const long long chunk = blockIdx.x;
  int lo = 0, hi = ntab - 1;
  while (lo < hi) {  // last entry with chunk0 <= chunk
    const int mid = (lo + hi + 1) >> 1;
    if (tab[mid].chunk0 <= chunk) lo = mid;
    else hi = mid - 1;
  }
  const AdamEntry e = tab[lo];
  const long long start = (chunk - e.chunk0) * kAdamChunk;
  const long long end = min(start + (long long)kAdamChunk, e.n);
  const float lr = *lr_ptr;
  const float decay = 1.f - lr * wd;
  for (long long i = start + threadIdx.x; i < end; i += blockDim.x) {
    const float g = e.g[i];
    float m = torch_lerp(e.m[i], g, one_m_b1);
    float v = torch_lerp(e.v[i], g * g, one_m_b2);
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

void adamw_multi(std::vector<torch::Tensor> params, std::vector<torch::Tensor> grads, std::vector<torch::Tensor> m,
                 std::vector<torch::Tensor> v, torch::Tensor lr, double beta1, double beta2, double eps, double wd,
                 std::vector<double> bc1, std::vector<double> bc2, bool cautious) {
  const int n = (int)params.size();
  TORCH_CHECK(n > 0 && grads.size() == (size_t)n && m.size() == (size_t)n && v.size() == (size_t)n, "table sizes");
  c10::cuda::CUDAGuard guard(params[0].device());
  std::vector<AdamEntry> host(n);
  long long chunks = 0;
  for (int i = 0; i < n; ++i) {
    for (auto* t : {&params[i], &grads[i], &m[i], &v[i]})
      TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous(), "adamw tensors: fp32 contiguous");
    host[i] = AdamEntry{params[i].data_ptr<float>(), grads[i].data_ptr<float>(), m[i].data_ptr<float>(),
                        v[i].data_ptr<float>(), params[i].numel(), (float)bc1[i], (float)bc2[i], chunks};
    chunks += (params[i].numel() + kAdamChunk - 1) / kAdamChunk;
  }
  auto tab = torch::empty({(long long)(n * sizeof(AdamEntry))}, torch::dtype(torch::kUInt8).pinned_memory(true));
  memcpy(tab.data_ptr(), host.data(), n * sizeof(AdamEntry));
  auto dtab = tab.to(params[0].device(), /*non_blocking=*/true);
  auto s = at::cuda::getCurrentCUDAStream();
  // `one minus beta` in float64 then rounded, like the Python float lerp weight.
  adamw_multi_kernel<<<(unsigned)chunks, 256, 0, s>>>(reinterpret_cast<const AdamEntry*>(dtab.data_ptr()), n,
                                                      lr.data_ptr<float>(), (float)(1.0 - beta1), (float)(1.0 - beta2),
                                                      (float)eps, (float)wd, cautious ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Muon apply (the reference's last line of the Muon step), elementwise over a stack:
//   t = bf16(bf16(lr) * g)          (0-dim fp32 lr times a bf16 g computes in bf16)
//   w = w - (t + lrwd * w * [g * w >= 0])
// Used by every rank on the gathered bf16 updates of distributed Muon.
__global__ void muon_apply_kernel(float* __restrict__ w, const __nv_bfloat16* __restrict__ g, long long n,
                                  const float* __restrict__ lr_ptr, const float* __restrict__ lrwd_ptr) {
  const float lr_b = __bfloat162float(__float2bfloat16_rn(*lr_ptr));
  const float lrwd = *lrwd_ptr;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float gv = __bfloat162float(g[i]);
    const float wv = w[i];
    const float t = __bfloat162float(__float2bfloat16_rn(lr_b * gv));
    const float mask = (gv * wv >= 0.f) ? 1.f : 0.f;  // bf16 g times fp32 w promotes to fp32
    w[i] = wv - (t + lrwd * wv * mask);
  }
}

void muon_apply(torch::Tensor w, torch::Tensor g, torch::Tensor lr, torch::Tensor lrwd) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kFloat && w.is_contiguous(), "w fp32 contiguous");
  TORCH_CHECK(g.scalar_type() == at::kBFloat16 && g.is_contiguous() && g.numel() == w.numel(), "g bf16 like w");
  c10::cuda::CUDAGuard guard(w.device());
  const long long n = w.numel();
  const int blocks = (int)std::min<long long>((n + 255) / 256, 148 * 16);
  muon_apply_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      w.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), n, lr.data_ptr<float>(),
      lrwd.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tfb
