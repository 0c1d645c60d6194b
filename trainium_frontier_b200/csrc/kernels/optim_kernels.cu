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

// ============================================================================ Muon owner math
// The part of the Muon step between the momentum prologue (muon_pre) and the apply, for a
// stack of K matrices [K, r, c] (reference train.py:3608-3647):
//   muon_fro_scale  x = x / d with d = bf16(bf16(bf16(||x||_F) * 1.01) + 1e-6): the
//                   reference's normalisation in its bf16 op order (norm rounded to bf16,
//                   each scalar op rounded, IEEE division), from the fp32 partial sums
//                   of squares muon_pre wrote (added here in a fixed order);
//   normuon_*       the NorMuon second moment on the Newton-Schulz output gq:
//                   v_mean = mean over the reduced dim of gq^2 (columns of a tall or
//                   square matrix, rows of a wide one); second = lerp(second, v_mean, 1-b2);
//                   step = rsqrt(max(second, 1e-10)); the update is
//                   gq * bf16(step * ||gq|| / max(||step * gq||, 1e-10)), the norms
//                   computed from v_mean as the reference does.
__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__global__ void muon_fro_scale_kernel(__nv_bfloat16* __restrict__ x, long long per, const float* __restrict__ fro,
                                      int nparts) {
  const int k = blockIdx.y;
  float ss = 0.f;
  for (int p = 0; p < nparts; ++p) ss += fro[(long long)k * nparts + p];  // fixed order
  const float nrm = bf16r(sqrtf(ss));
  const float d = bf16r(bf16r(nrm * 1.01f) + 1e-6f);
  uint4* xv = reinterpret_cast<uint4*>(x + (long long)k * per);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < per / 8; i += (long long)gridDim.x * blockDim.x) {
    uint4 u = xv[i];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      h[j] = __floats2bfloat162_rn(__fdiv_rn(f.x, d), __fdiv_rn(f.y, d));
    }
    xv[i] = u;
  }
}

// tall (r >= c): vmean[k, i] = sum_j gq[k, i, j]^2 / c, one warp per row.
__global__ void normuon_vmean_rows_kernel(const __nv_bfloat16* __restrict__ gq, int r, int c, float* __restrict__ vmean) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + warp;  // over K * r
  const int k = blockIdx.y;
  if (row >= r) return;
  const __nv_bfloat16* src = gq + ((long long)k * r + row) * c;
  float ss = 0.f;
  for (int j = lane * 8; j < c; j += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + j);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(h[q]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) vmean[(long long)k * r + row] = ss / (float)c;
}

// wide (r < c): vmean[k, j] = sum_i gq[k, i, j]^2 / r; a block is 32 columns x 8 row slices.
__global__ void normuon_vmean_cols_kernel(const __nv_bfloat16* __restrict__ gq, int r, int c, float* __restrict__ vmean) {
  const int k = blockIdx.y;
  const int col = blockIdx.x * 32 + (threadIdx.x & 31);
  const int slice = threadIdx.x >> 5;
  __shared__ float part[8][33];
  float ss = 0.f;
  if (col < c) {
    const __nv_bfloat16* src = gq + (long long)k * r * c + col;
    for (int i = slice; i < r; i += 8) {
      const float f = __bfloat162float(src[(long long)i * c]);
      ss += f * f;
    }
  }
  part[slice][threadIdx.x & 31] = ss;
  __syncthreads();
  if (slice == 0 && col < c) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) t += part[q][threadIdx.x & 31];
    vmean[(long long)k * c + col] = t / (float)r;
  }
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) t += red[w];
  return t;
}

// one block per matrix: second moment update and the per-row / per-column bf16 scale
__global__ void normuon_scale_kernel(const float* __restrict__ vmean, float* __restrict__ second, int L, float red,
                                     const float* __restrict__ one_b2_ptr, float* __restrict__ scale) {
  constexpr int NT = 1024;
  __shared__ float redbuf[NT / 32];
  const int k = blockIdx.x;
  const float* vm = vmean + (long long)k * L;
  float* sec = second + (long long)k * L;
  float* sc = scale + (long long)k * L;
  const float w = *one_b2_ptr;
  float vsum = 0.f, ssum = 0.f;
  for (int i = threadIdx.x; i < L; i += NT) {
    const float v = vm[i];
    const float a = sec[i];
    const float snew = (fabsf(w) < 0.5f) ? a + w * (v - a) : v - (v - a) * (1.f - w);
    sec[i] = snew;
    const float st = rsqrtf(fmaxf(snew, 1e-10f));
    sc[i] = st;
    vsum += v;
    ssum += (v * red) * (st * st);
  }
  const float vt = block_sum<NT>(vsum, redbuf);
  const float stot = block_sum<NT>(ssum, redbuf);
  const float v_norm = sqrtf(vt * red);
  const float q = v_norm / fmaxf(sqrtf(stot), 1e-10f);
  for (int i = threadIdx.x; i < L; i += NT) sc[i] = bf16r(sc[i] * q);
}

// out = bf16(gq * scale[row or col]); with w != null the update is applied to the fp32
// masters instead (w -= bf16(bf16(lr) * u) + lrwd * w * [u * w >= 0], the apply of
// muon_apply) and out is not written.
__global__ void normuon_apply_kernel(const __nv_bfloat16* __restrict__ gq, const float* __restrict__ scale, int r,
                                     int c, int tall, long long total, __nv_bfloat16* __restrict__ out,
                                     float* __restrict__ w, const float* __restrict__ lr_ptr,
                                     const float* __restrict__ lrwd_ptr) {
  const float lr_b = w ? bf16r(*lr_ptr) : 0.f;
  const float lrwd = w ? *lrwd_ptr : 0.f;
  const long long per = (long long)r * c;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < total / 8; v += (long long)gridDim.x * blockDim.x) {
    const long long e = v * 8;
    const long long k = e / per;
    const long long rem = e - k * per;
    const int i = (int)(rem / c), j = (int)(rem - (long long)i * c);
    const uint4 u = *reinterpret_cast<const uint4*>(gq + e);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
    float g8[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 f = __bfloat1622float2(h[q]);
      g8[2 * q] = f.x;
      g8[2 * q + 1] = f.y;
    }
    const float* srow = scale + k * (tall ? r : c);
#pragma unroll
    for (int q = 0; q < 8; ++q) g8[q] = bf16r(g8[q] * (tall ? srow[i] : srow[j + q]));
    if (w == nullptr) {
      uint4 o;
      o.x = pack_bf16x2(g8[0], g8[1]);
      o.y = pack_bf16x2(g8[2], g8[3]);
      o.z = pack_bf16x2(g8[4], g8[5]);
      o.w = pack_bf16x2(g8[6], g8[7]);
      *reinterpret_cast<uint4*>(out + e) = o;
    } else {
      float4* wp = reinterpret_cast<float4*>(w + e);
      float4 w0 = wp[0], w1 = wp[1];
      float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float t = bf16r(lr_b * g8[q]);
        const float mask = (g8[q] * wv[q] >= 0.f) ? 1.f : 0.f;
        wv[q] = wv[q] - (t + lrwd * wv[q] * mask);
      }
      wp[0] = make_float4(wv[0], wv[1], wv[2], wv[3]);
      wp[1] = make_float4(wv[4], wv[5], wv[6], wv[7]);
    }
  }
}

// fro: fp32 [K, P] partial sums of squares per matrix (muon_pre's), added in order.
void muon_fro_scale(torch::Tensor x, torch::Tensor fro) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 3 && x.is_contiguous(), "x bf16 [K, r, c]");
  TORCH_CHECK(fro.scalar_type() == at::kFloat && fro.dim() == 2 && fro.size(0) == x.size(0) && fro.is_contiguous(),
              "fro fp32 [K, P]");
  const long long per = x.size(1) * x.size(2);
  TORCH_CHECK(per % 8 == 0, "matrix size % 8");
  c10::cuda::CUDAGuard guard(x.device());
  dim3 grid((unsigned)std::max<long long>(1, std::min<long long>((per / 8 + 255) / 256, 64)), (unsigned)x.size(0));
  muon_fro_scale_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), per, fro.data_ptr<float>(), (int)fro.size(1));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// gq [K, r, c] bf16; second fp32 [K, r, 1] (tall or square) or [K, 1, c] (wide);
// out bf16 like gq, or (w, lr, lrwd) to apply the update to the fp32 masters in place.
void normuon_tail(torch::Tensor gq, torch::Tensor second, torch::Tensor one_b2, c10::optional<torch::Tensor> out,
                  c10::optional<torch::Tensor> w, c10::optional<torch::Tensor> lr, c10::optional<torch::Tensor> lrwd) {
  TORCH_CHECK(gq.is_cuda() && gq.scalar_type() == at::kBFloat16 && gq.dim() == 3 && gq.is_contiguous(), "gq bf16 [K, r, c]");
  const int K = (int)gq.size(0), r = (int)gq.size(1), c = (int)gq.size(2);
  const bool tall = r >= c;
  const int L = tall ? r : c;
  TORCH_CHECK(second.scalar_type() == at::kFloat && second.is_contiguous() && second.numel() == (long long)K * L,
              "second moment fp32 with one entry per kept row / column");
  TORCH_CHECK(c % 8 == 0, "columns % 8");
  TORCH_CHECK(out.has_value() != w.has_value(), "exactly one of out / w");
  c10::cuda::CUDAGuard guard(gq.device());
  auto s = at::cuda::getCurrentCUDAStream();
  auto vmean = torch::empty({(long long)K * L}, gq.options().dtype(torch::kFloat));
  auto scale = torch::empty({(long long)K * L}, gq.options().dtype(torch::kFloat));
  const auto* gp = reinterpret_cast<const __nv_bfloat16*>(gq.data_ptr());
  if (tall) {
    normuon_vmean_rows_kernel<<<dim3((unsigned)((r + 7) / 8), (unsigned)K), 256, 0, s>>>(gp, r, c, vmean.data_ptr<float>());
  } else {
    normuon_vmean_cols_kernel<<<dim3((unsigned)((c + 31) / 32), (unsigned)K), 256, 0, s>>>(gp, r, c, vmean.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  normuon_scale_kernel<<<(unsigned)K, 1024, 0, s>>>(vmean.data_ptr<float>(), second.data_ptr<float>(), L,
                                                    (float)(tall ? c : r), one_b2.data_ptr<float>(),
                                                    scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const long long total = (long long)K * r * c;
  const int blocks = (int)std::min<long long>((total / 8 + 255) / 256, 148 * 8);
  if (w.has_value()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && w->is_contiguous() && w->numel() == total, "w fp32 like gq");
    TORCH_CHECK(lr.has_value() && lrwd.has_value(), "lr / lrwd device scalars");
    normuon_apply_kernel<<<blocks, 256, 0, s>>>(gp, scale.data_ptr<float>(), r, c, tall ? 1 : 0, total, nullptr,
                                                w->data_ptr<float>(), lr->data_ptr<float>(), lrwd->data_ptr<float>());
  } else {
    TORCH_CHECK(out->scalar_type() == at::kBFloat16 && out->is_contiguous() && out->numel() == total, "out bf16 like gq");
    normuon_apply_kernel<<<blocks, 256, 0, s>>>(gp, scale.data_ptr<float>(), r, c, tall ? 1 : 0, total,
                                                reinterpret_cast<__nv_bfloat16*>(out->data_ptr()), nullptr, nullptr,
                                                nullptr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tfb
