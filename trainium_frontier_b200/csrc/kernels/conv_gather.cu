// Two memory-bound ops of the model family's optional features:
//
//  * causal depthwise conv1d (the block's local conv and Engram's conv):
//      y[b, t, c] = sum_{k<K} w[c, k] * x[b, t - (K-1) + k, c]      (x = 0 before t = 0)
//    Forward: a thread owns 8 channels (one 16-byte vector) and a run of time steps,
//    keeping the K-1 previous inputs in registers, so every input is read once.
//    Backward: the same walk over dy produces dx, and each thread's fp32 partial sums
//    of dw are written to a per-run slot; a second kernel adds the slots in a fixed
//    order, so dw is bitwise reproducible.
//  * hashed n-gram embedding lookup: the row id of every position is computed from the
//    token and its one or two predecessors (products with layer primes, XOR, modulo the
//    table's prime row count; a missing predecessor is the pad id), and the row is
//    gathered and cast to bf16 in the same kernel (one warp per position).  The backward
//    adds each position's gradient row into the fp32 table gradient with vector atomics.
//
// Reference counterparts: CausalConv (train.py:1316-1329) and its research kernel
// (research/scratch/causal_conv_dev2.py:144-324); the n-gram hashing / lookup
// (train.py:3087-3140) and its research gather kernel
// (research/scratch/nki_ngram_gather_dev.py:119-143).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

namespace {

constexpr int kConvRun = 64;    // time steps per thread
constexpr int kConvMaxK = 8;

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  u.x = pack_bf16x2(f[0], f[1]);
  u.y = pack_bf16x2(f[2], f[3]);
  u.z = pack_bf16x2(f[4], f[5]);
  u.w = pack_bf16x2(f[6], f[7]);
  return u;
}

// grid (ceil(C/8 / blockDim), ceil(T / kConvRun), B); w: [C][K] fp32 (rounded to bf16 in
// use, as the reference casts the weight to the activation dtype).
template <int K>
__global__ void causal_conv_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                       __nv_bfloat16* __restrict__ y, int T, int C) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 * 8 >= C) return;
  const int t0 = blockIdx.y * kConvRun;
  const long long base = (long long)blockIdx.z * T * C + c8 * 8;
  float wk[K][8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k][j] = __bfloat162float(__float2bfloat16_rn(w[(c8 * 8 + j) * K + k]));
  float hist[K][8];  // hist[k] = x[t - (K-1) + k]
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 - (K - 1) + k;
    if (t >= 0) unpack8(*reinterpret_cast<const uint4*>(x + base + (long long)t * C), hist[k]);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) hist[k][j] = 0.f;
  }
  const int t1 = min(T, t0 + kConvRun);
  for (int t = t0; t < t1; ++t) {
    unpack8(*reinterpret_cast<const uint4*>(x + base + (long long)t * C), hist[K - 1]);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) s = fmaf(wk[k][j], hist[k][j], s);
      o[j] = s;
    }
    *reinterpret_cast<uint4*>(y + base + (long long)t * C) = pack8(o);
#pragma unroll
    for (int k = 0; k < K - 1; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) hist[k][j] = hist[k + 1][j];
  }
}

// dx[t] = sum_k w[k] dy[t + (K-1) - k]; dw partial[run][c][k] = sum_t dy[t] x[t - (K-1) + k].
template <int K>
__global__ void causal_conv_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                       const float* __restrict__ w, __nv_bfloat16* __restrict__ dx,
                                       float* __restrict__ dw_part, int T, int C) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 * 8 >= C) return;
  const int t0 = blockIdx.y * kConvRun;
  const long long base = (long long)blockIdx.z * T * C + c8 * 8;
  float wk[K][8];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) wk[k][j] = __bfloat162float(__float2bfloat16_rn(w[(c8 * 8 + j) * K + k]));
  // xh[k] = x[t - (K-1) + k] for the dw sums; gf[k] = dy[t + k] for dx
  float xh[K][8], gf[K][8], acc[K][8];
#pragma unroll
  for (int k = 0; k < K; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 - (K - 1) + k;
    if (t >= 0) unpack8(*reinterpret_cast<const uint4*>(x + base + (long long)t * C), xh[k]);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) xh[k][j] = 0.f;
  }
#pragma unroll
  for (int k = 0; k < K - 1; ++k) {
    const int t = t0 + k;
    if (t < T) unpack8(*reinterpret_cast<const uint4*>(dy + base + (long long)t * C), gf[k + 1]);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) gf[k + 1][j] = 0.f;
  }
  const int t1 = min(T, t0 + kConvRun);
  for (int t = t0; t < t1; ++t) {
    // shift dy window: gf[k] = dy[t + k]
#pragma unroll
    for (int k = 0; k < K - 1; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) gf[k][j] = gf[k + 1][j];
    if (t + K - 1 < T) unpack8(*reinterpret_cast<const uint4*>(dy + base + (long long)(t + K - 1) * C), gf[K - 1]);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) gf[K - 1][j] = 0.f;
    unpack8(*reinterpret_cast<const uint4*>(x + base + (long long)t * C), xh[K - 1]);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < K; ++k) s = fmaf(wk[k][j], gf[K - 1 - k][j], s);
      o[j] = s;
#pragma unroll
      for (int k = 0; k < K; ++k) acc[k][j] = fmaf(gf[0][j], xh[k][j], acc[k][j]);
    }
    *reinterpret_cast<uint4*>(dx + base + (long long)t * C) = pack8(o);
#pragma unroll
    for (int k = 0; k < K - 1; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) xh[k][j] = xh[k + 1][j];
  }
  const long long run = (long long)blockIdx.z * gridDim.y + blockIdx.y;
  float* dst = dw_part + run * C * K + (long long)c8 * 8 * K;
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int k = 0; k < K; ++k) dst[j * K + k] = acc[k][j];
}

// dw[i] (+)= sum over runs r (in order) of part[r][i]; one thread per weight element.
__global__ void conv_dw_reduce_kernel(const float* __restrict__ part, int runs, int n, float* __restrict__ dw,
                                      int accumulate) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int r = 0; r < runs; ++r) s += part[(long long)r * n + i];
  dw[i] = accumulate ? dw[i] + s : s;
}

// ---------------------------------------------------------------------------- n-gram
struct NgramHash {
  long long p1, p2, p3, mod, pad;
  int order;  // 2 (bigram) or 3 (trigram)
};

__device__ __forceinline__ long long ngram_row(const int* __restrict__ idx, int t, long long cur_off, const NgramHash& h) {
  const long long cur = idx[cur_off];
  const long long prev = t >= 1 ? (long long)idx[cur_off - 1] : h.pad;
  long long v;
  if (h.order == 2) {
    v = (prev * h.p1) ^ (cur * h.p2);
  } else {
    const long long prev2 = t >= 2 ? (long long)idx[cur_off - 2] : h.pad;
    v = (prev2 * h.p1) ^ (prev * h.p2) ^ (cur * h.p3);
  }
  return v % h.mod;
}

// One warp per position: row id from the hash, then the row (Dn values) gathered and cast.
template <typename TT>
__global__ void ngram_gather_kernel(const int* __restrict__ idx, int T, long long n_pos, NgramHash h,
                                    const TT* __restrict__ table, int Dn, __nv_bfloat16* __restrict__ out,
                                    int* __restrict__ rows_out) {
  const long long pos = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pos >= n_pos) return;
  const int t = (int)(pos % T);
  const long long row = ngram_row(idx, t, pos, h);
  if (lane == 0 && rows_out) rows_out[pos] = (int)row;
  const TT* src = table + row * Dn;
  __nv_bfloat16* dst = out + pos * Dn;
  for (int j = lane * 4; j < Dn; j += 128) {
    float f[4];
    if constexpr (sizeof(TT) == 4) {
      const float4 v = *reinterpret_cast<const float4*>(src + j);
      f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w;
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(src + j);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
      f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    }
    uint2 o;
    o.x = pack_bf16x2(f[0], f[1]);
    o.y = pack_bf16x2(f[2], f[3]);
    *reinterpret_cast<uint2*>(dst + j) = o;
  }
}

// grad[rows[pos]] += dout[pos] (fp32 vector atomics); one warp per position.
__global__ void ngram_scatter_kernel(const int* __restrict__ rows, long long n_pos, const __nv_bfloat16* __restrict__ dout,
                                     int Dn, float* __restrict__ grad) {
  const long long pos = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (pos >= n_pos) return;
  float* dst = grad + (long long)rows[pos] * Dn;
  const __nv_bfloat16* src = dout + pos * Dn;
  for (int j = lane * 4; j < Dn; j += 128) {
    const uint2 u = *reinterpret_cast<const uint2*>(src + j);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    atomicAdd(reinterpret_cast<float4*>(dst + j), make_float4(a.x, a.y, b.x, b.y));
  }
}

}  // namespace

// ---------------------------------------------------------------------------- host
static void check_conv(const torch::Tensor& x, const torch::Tensor& w, int64_t& B, int64_t& T, int64_t& Cc, int& K) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 3 && x.is_contiguous(),
              "causal conv: x must be contiguous bf16 [B, T, C]");
  B = x.size(0); T = x.size(1); Cc = x.size(2);
  TORCH_CHECK(Cc % 8 == 0, "causal conv: C must be a multiple of 8");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == at::kFloat && w.is_contiguous() && w.numel() % Cc == 0,
              "causal conv: w must be contiguous fp32 [C, 1, K]");
  K = (int)(w.numel() / Cc);
  TORCH_CHECK(K >= 1 && K <= kConvMaxK, "causal conv: kernel size 1..8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0, "causal conv: x must be 16-byte aligned");
}

#define TFB_CONV_K(K, ...)                                   \
  switch (K) {                                               \
    case 1: { constexpr int KK = 1; __VA_ARGS__; break; }     \
    case 2: { constexpr int KK = 2; __VA_ARGS__; break; }     \
    case 3: { constexpr int KK = 3; __VA_ARGS__; break; }     \
    case 4: { constexpr int KK = 4; __VA_ARGS__; break; }     \
    case 5: { constexpr int KK = 5; __VA_ARGS__; break; }     \
    case 6: { constexpr int KK = 6; __VA_ARGS__; break; }     \
    case 7: { constexpr int KK = 7; __VA_ARGS__; break; }     \
    case 8: { constexpr int KK = 8; __VA_ARGS__; break; }     \
    default: TORCH_CHECK(false, "kernel size");               \
  }

void causal_conv_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor y) {
  int64_t B, T, Cc;
  int K;
  check_conv(x, w, B, T, Cc, K);
  TORCH_CHECK(y.sizes() == x.sizes() && y.is_contiguous() && y.scalar_type() == at::kBFloat16, "y like x");
  c10::cuda::CUDAGuard guard(x.device());
  const int c8 = (int)(Cc / 8);
  const int threads = std::min(256, ((c8 + 31) / 32) * 32);
  dim3 grid((c8 + threads - 1) / threads, (unsigned)((T + kConvRun - 1) / kConvRun), (unsigned)B);
  auto s = at::cuda::getCurrentCUDAStream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  TFB_CONV_K(K, causal_conv_fwd_kernel<KK><<<grid, threads, 0, s>>>(xp, w.data_ptr<float>(), yp, (int)T, (int)Cc));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dx (bf16, like x) and dw (fp32 [C*K], overwritten or accumulated); part: fp32 scratch of
// at least B * ceil(T / 64) * C * K elements.
void causal_conv_bwd(torch::Tensor x, torch::Tensor w, torch::Tensor dy, torch::Tensor dx, torch::Tensor dw,
                     torch::Tensor part, bool accumulate) {
  int64_t B, T, Cc;
  int K;
  check_conv(x, w, B, T, Cc, K);
  TORCH_CHECK(dy.sizes() == x.sizes() && dy.is_contiguous() && dy.scalar_type() == at::kBFloat16, "dy like x");
  TORCH_CHECK(dx.sizes() == x.sizes() && dx.is_contiguous() && dx.scalar_type() == at::kBFloat16, "dx like x");
  TORCH_CHECK(dw.scalar_type() == at::kFloat && dw.is_contiguous() && dw.numel() == Cc * K, "dw fp32 [C*K]");
  const int64_t runs = B * ((T + kConvRun - 1) / kConvRun);
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.numel() >= runs * Cc * K, "dw partial scratch too small");
  c10::cuda::CUDAGuard guard(x.device());
  const int c8 = (int)(Cc / 8);
  const int threads = std::min(256, ((c8 + 31) / 32) * 32);
  dim3 grid((c8 + threads - 1) / threads, (unsigned)((T + kConvRun - 1) / kConvRun), (unsigned)B);
  auto s = at::cuda::getCurrentCUDAStream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  const auto* gp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto* dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  TFB_CONV_K(K, causal_conv_bwd_kernel<KK><<<grid, threads, 0, s>>>(xp, gp, w.data_ptr<float>(), dxp,
                                                                    part.data_ptr<float>(), (int)T, (int)Cc));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int n = (int)(Cc * K);
  conv_dw_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(part.data_ptr<float>(), (int)runs, n, dw.data_ptr<float>(),
                                                        accumulate ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// out[pos] = bf16(table[row(pos)]), rows[pos] = row(pos) for idx [B, T] int32.
void ngram_gather(torch::Tensor idx, int64_t order, int64_t p1, int64_t p2, int64_t p3, int64_t mod, int64_t pad,
                  torch::Tensor table, torch::Tensor out, torch::Tensor rows) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.dim() == 2 && idx.is_contiguous(),
              "ngram: idx contiguous int32 [B, T]");
  TORCH_CHECK(order == 2 || order == 3, "ngram order 2 or 3");
  TORCH_CHECK(table.dim() == 2 && table.is_contiguous() &&
                  (table.scalar_type() == at::kFloat || table.scalar_type() == at::kBFloat16),
              "ngram: table contiguous fp32 / bf16 [R, Dn]");
  const int64_t Dn = table.size(1), n_pos = idx.numel();
  TORCH_CHECK(Dn % 4 == 0 && mod >= 1 && mod <= table.size(0), "ngram: Dn % 4 == 0, mod <= rows");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == n_pos * Dn, "ngram: out bf16");
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.is_contiguous() && rows.numel() == n_pos, "ngram: rows int32");
  c10::cuda::CUDAGuard guard(idx.device());
  NgramHash h{p1, p2, p3, mod, pad, (int)order};
  const int warps = 8;
  const unsigned blocks = (unsigned)((n_pos + warps - 1) / warps);
  auto s = at::cuda::getCurrentCUDAStream();
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (table.scalar_type() == at::kFloat)
    ngram_gather_kernel<float><<<blocks, warps * 32, 0, s>>>(idx.data_ptr<int>(), (int)idx.size(1), n_pos, h,
                                                             table.data_ptr<float>(), (int)Dn, op, rows.data_ptr<int>());
  else
    ngram_gather_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, s>>>(
        idx.data_ptr<int>(), (int)idx.size(1), n_pos, h, reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
        (int)Dn, op, rows.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void ngram_scatter(torch::Tensor rows, torch::Tensor dout, torch::Tensor grad) {
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.is_contiguous(), "rows int32");
  TORCH_CHECK(grad.scalar_type() == at::kFloat && grad.is_contiguous() && grad.dim() == 2, "grad fp32 [R, Dn]");
  const int64_t Dn = grad.size(1), n_pos = rows.numel();
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.is_contiguous() && dout.numel() == n_pos * Dn, "dout bf16");
  TORCH_CHECK(Dn % 4 == 0 && (reinterpret_cast<uintptr_t>(grad.data_ptr()) & 15) == 0, "16-byte aligned rows");
  c10::cuda::CUDAGuard guard(rows.device());
  const int warps = 8;
  const unsigned blocks = (unsigned)((n_pos + warps - 1) / warps);
  ngram_scatter_kernel<<<blocks, warps * 32, 0, at::cuda::getCurrentCUDAStream()>>>(
      rows.data_ptr<int>(), n_pos, reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), (int)Dn,
      grad.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tfb
