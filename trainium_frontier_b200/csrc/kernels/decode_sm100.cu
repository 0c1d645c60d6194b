// Inference kernels for KV-cache decoding (one new token per sequence per step).
//
// decode_attn: single-query attention over a KV cache laid out like the projection
// buffers, [B, T_max, H*D] (head h at columns h*D), valid length read from device
// memory so a whole decode step can be captured once in a CUDA graph and replayed.
//   one CTA (128 threads) per (batch, head):
//   phase 1  thread-per-key scores q.k (16-byte loads of the key row) into shared
//            memory, block max / sum of exp;
//   phase 2  thread-per-dimension output o[d] = sum_k p_k v_k[d] / l (coalesced rows).
// kv_append: writes this step's k and v rows into the caches at the device-side
// position; step_advance: increments the device-side position / length counters.
// The reference has no decode path; the attention is the math of train.py:2564-2567 over a
// key/value cache.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

constexpr int kDecThreads = 128;

template <int D>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(
    const __nv_bfloat16* __restrict__ q, long long ldq, const __nv_bfloat16* __restrict__ kc,
    const __nv_bfloat16* __restrict__ vc, long long cache_ld, long long cache_bstride, const int* __restrict__ len_ptr,
    int len_max, __nv_bfloat16* __restrict__ out, long long ldo, int H, float scale) {
  extern __shared__ float s_scores[];
  __shared__ float red[kDecThreads / 32];
  __shared__ __align__(16) float s_q[D];
  const int bh = blockIdx.x;
  const int b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  int L = *len_ptr;
  L = L < 1 ? 1 : (L > len_max ? len_max : L);
  for (int d = tid; d < D; d += kDecThreads) s_q[d] = __bfloat162float(q[(long long)b * ldq + h * D + d]) * scale;
  __syncthreads();
  const __nv_bfloat16* kb = kc + (long long)b * cache_bstride + h * D;
  const __nv_bfloat16* vb = vc + (long long)b * cache_bstride + h * D;
  float mx = -INFINITY;
  for (int k = tid; k < L; k += kDecThreads) {
    const uint4* kr = reinterpret_cast<const uint4*>(kb + (long long)k * cache_ld);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      const uint4 u = kr[c];
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h2[j]);
        acc += f.x * s_q[c * 8 + 2 * j] + f.y * s_q[c * 8 + 2 * j + 1];
      }
    }
    s_scores[k] = acc;
    mx = fmaxf(mx, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kDecThreads / 32; ++w) m = fmaxf(m, red[w]);
  __syncthreads();
  float sum = 0.f;
  for (int k = tid; k < L; k += kDecThreads) {
    const float p = __expf(s_scores[k] - m);
    s_scores[k] = p;
    sum += p;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((tid & 31) == 0) red[tid >> 5] = sum;
  __syncthreads();
  float l = 0.f;
#pragma unroll
  for (int w = 0; w < kDecThreads / 32; ++w) l += red[w];
  const float inv_l = 1.f / l;
  for (int d = tid; d < D; d += kDecThreads) {
    float acc = 0.f;
    for (int k = 0; k < L; ++k) acc += s_scores[k] * __bfloat162float(vb[(long long)k * cache_ld + d]);
    out[(long long)b * ldo + h * D + d] = __float2bfloat16_rn(acc * inv_l);
  }
}

// decode_attn_split: the same attention with the cache length split over `splits` CTAs per
// (batch, head) so the KV stream is read by many SMs at once.  The cache is addressed by
// strides (batch, head, token), so it may be stored token-major ([B, T_max, H*D], the
// projection buffer's layout) or head-major ([B, H, T_max, D], each (batch, head) one
// contiguous stream).  Each warp scores two keys per load (a half-warp per key, 16 bytes
// per lane: dims 8l .. 8l+7), eight keys per iteration with every K and V load of the
// eight issued before any math; a CTA keeps an unnormalised partial output plus (max, sum)
// in a workspace, and the last CTA of its (batch, head) -- an arrival counter -- combines
// the partials in split order, writes the row and re-zeroes the counter (no memset
// between graph replays).
template <int D>
__global__ void __launch_bounds__(kDecThreads) decode_attn_split_kernel(
    const __nv_bfloat16* __restrict__ q, long long ldq, const __nv_bfloat16* __restrict__ kc,
    const __nv_bfloat16* __restrict__ vc, long long cs_b, long long cs_h, long long cs_t,
    const int* __restrict__ len_ptr, int len_max, __nv_bfloat16* __restrict__ out, long long ldo, int H, float scale,
    int splits, float* __restrict__ ws, int* __restrict__ cnt) {
  static_assert(D == 128, "a half-warp covers the 128 dims, 8 per lane");
  // partial record = D outputs + (max, sum), padded to a multiple of 4 floats so every
  // record starts on a 16-byte boundary (float4 stores / loads)
  constexpr int kPartStride = D + 4;
  constexpr int NW = kDecThreads / 32;
  constexpr int KPH = 4;            // keys per half-warp per iteration
  constexpr int KPW = 2 * KPH;      // keys per warp per iteration
  __shared__ float s_m[NW], s_l[NW];
  __shared__ __align__(16) float s_o[NW][D];
  __shared__ int s_last;
  const int bh = blockIdx.x / splits, sp = blockIdx.x % splits;
  const int b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  // launched as a programmatic dependent of the QKV projection: wait for its q / cache
  // writes, and let the next projection start streaming its weights meanwhile
  griddep_wait();
  griddep_launch_dependents();
  int L = *len_ptr;
  L = L < 1 ? 1 : (L > len_max ? len_max : L);
  const int chunk = (L + splits - 1) / splits;
  const int k0 = sp * chunk, k1 = min(L, k0 + chunk);
  // q slice of this lane (dims 8*hl .. 8*hl+7), pre-scaled
  float qs[8];
  {
    const uint4 qu = *reinterpret_cast<const uint4*>(q + (long long)b * ldq + h * D + 8 * hl);
    const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qu);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(q2[i]);
      qs[2 * i] = f.x * scale;
      qs[2 * i + 1] = f.y * scale;
    }
  }
  const __nv_bfloat16* kb = kc + (long long)b * cs_b + (long long)h * cs_h + 8 * hl;
  const __nv_bfloat16* vb = vc + (long long)b * cs_b + (long long)h * cs_h + 8 * hl;
  float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  for (int kw = k0 + warp * KPW; kw < k1; kw += NW * KPW) {
    // this half-warp's keys: kw + half + 2 * j
    uint4 ku[KPH], vu[KPH];
#pragma unroll
    for (int j = 0; j < KPH; ++j) {
      const int k = min(kw + half + 2 * j, k1 - 1);  // clamped: past-the-end keys are masked below
      ku[j] = *reinterpret_cast<const uint4*>(kb + (long long)k * cs_t);
      vu[j] = *reinterpret_cast<const uint4*>(vb + (long long)k * cs_t);
    }
    float sd[KPH];
#pragma unroll
    for (int j = 0; j < KPH; ++j) {
      const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&ku[j]);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(k2[i]);
        acc += qs[2 * i] * f.x + qs[2 * i + 1] * f.y;
      }
      sd[j] = acc;
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1)
#pragma unroll
      for (int j = 0; j < KPH; ++j) sd[j] += __shfl_xor_sync(0xffffffffu, sd[j], off);
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < KPH; ++j) {
      if (kw + half + 2 * j >= k1) sd[j] = -INFINITY;
      mx = fmaxf(mx, sd[j]);
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));  // one running max per warp
    mx = fmaxf(mx, m);
    const float corr = __expf(m - mx);
    l *= corr;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] *= corr;
#pragma unroll
    for (int j = 0; j < KPH; ++j) {
      const float p = __expf(sd[j] - mx);
      const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&vu[j]);
      l += p;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(v2[i]);
        o[2 * i] += p * f.x;
        o[2 * i + 1] += p * f.y;
      }
    }
    m = mx;
  }
  // the two half-warps share the running max: add their sums and outputs
  l += __shfl_xor_sync(0xffffffffu, l, 16);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] += __shfl_xor_sync(0xffffffffu, o[i], 16);
  // combine the warps of this CTA
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
  if (half == 0) {
    *reinterpret_cast<float4*>(&s_o[warp][8 * hl]) = make_float4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<float4*>(&s_o[warp][8 * hl + 4]) = make_float4(o[4], o[5], o[6], o[7]);
  }
  __syncthreads();
  float* part = ws + ((long long)bh * splits + sp) * kPartStride;
  if (warp == 0) {
    float M = s_m[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) M = fmaxf(M, s_m[w]);
    float Lsum = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = s_m[w] == -INFINITY ? 0.f : __expf(s_m[w] - M);
      Lsum += f * s_l[w];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += f * s_o[w][4 * lane + j];
    }
    *reinterpret_cast<float4*>(part + 4 * lane) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (lane == 0) {
      part[D] = M;
      part[D + 1] = Lsum;
    }
    __threadfence();
    __syncwarp();
    if (lane == 0) s_last = atomicAdd(cnt + bh, 1) == splits - 1;
  }
  __syncthreads();
  if (!s_last) return;
  // last split of this (batch, head): combine every split's partial
  if (warp == 0) {
    __threadfence();
    const float* base = ws + (long long)bh * splits * kPartStride;
    float M = -INFINITY;
    for (int t = 0; t < splits; ++t) M = fmaxf(M, __ldcg(base + t * kPartStride + D));
    float Lsum = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int t = 0; t < splits; ++t) {
      const float mt = __ldcg(base + t * kPartStride + D);
      const float f = mt == -INFINITY ? 0.f : __expf(mt - M);
      Lsum += f * __ldcg(base + t * kPartStride + D + 1);
      const float4 ot = __ldcg(reinterpret_cast<const float4*>(base + t * kPartStride + 4 * lane));
      acc[0] += f * ot.x; acc[1] += f * ot.y; acc[2] += f * ot.z; acc[3] += f * ot.w;
    }
    const float inv = 1.f / Lsum;
    uint2 u;
    u.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
    u.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<uint2*>(out + (long long)b * ldo + h * D + 4 * lane) = u;
    if (lane == 0) cnt[bh] = 0;
  }
}

// cache[b, pos, :] = src[b, :] for k and v (pos read from device memory).
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ ksrc, long long ldk,
                                 const __nv_bfloat16* __restrict__ vsrc, long long ldv, __nv_bfloat16* __restrict__ kc,
                                 __nv_bfloat16* __restrict__ vc, long long cache_ld, long long cache_bstride,
                                 const int* __restrict__ pos_ptr, int len_max, int B, int C) {
  const int pos = *pos_ptr;
  if (pos < 0 || pos >= len_max) return;
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i >= (long long)B * C) return;
  const int b = (int)(i / C), c = (int)(i % C);
  const long long dst = (long long)b * cache_bstride + (long long)pos * cache_ld + c;
  *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(ksrc + (long long)b * ldk + c);
  *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(vsrc + (long long)b * ldv + c);
}

// counters[0] = position of the next token, counters[1] = valid cache length.
__global__ void step_advance_kernel(int* counters) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    counters[0] += 1;
    counters[1] += 1;
  }
}

// Greedy pick over softcapped logits: argmax of the first V columns of bf16 rows; writes
// the token into idx_out[b] and into tokens[b * ld_tok + (counters[0] - start)].
__global__ void argmax_rows_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int V,
                                   int* __restrict__ idx_out, int* __restrict__ tokens, long long ld_tok,
                                   const int* __restrict__ counters, int start, int max_new) {
  const int b = blockIdx.x;
  const __nv_bfloat16* row = logits + (long long)b * ld;
  float best = -INFINITY;
  int arg = 0;
  const bool vec = (V % 8) == 0 && (ld % 8) == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0;
  if (vec) {  // 16-byte loads, all of a thread's loads issued before the compares
    constexpr int U = 4;
    for (int base = threadIdx.x * 8; base < V; base += blockDim.x * 8 * U) {
      uint4 u[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int j = base + k * blockDim.x * 8;
        u[k] = j < V ? *reinterpret_cast<const uint4*>(row + j) : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int j = base + k * blockDim.x * 8;
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u[k]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float v = __bfloat162float(e[i]);
          if (v > best) { best = v; arg = j + i; }
        }
      }
    }
  } else {
    for (int j = threadIdx.x; j < V; j += blockDim.x) {
      const float v = __bfloat162float(row[j]);
      if (v > best) { best = v; arg = j; }
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, arg, o);
    if (ov > best || (ov == best && oi < arg)) { best = ov; arg = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = arg; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > best || (sv[w] == best && si[w] < arg)) { best = sv[w]; arg = si[w]; }
    idx_out[b] = arg;
    const int slot = counters[0] - start;
    if (tokens && slot >= 0 && slot < max_new) tokens[(long long)b * ld_tok + slot] = arg;
  }
}

void decode_attn(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache, torch::Tensor len, int64_t H,
                 int64_t D, double scale, torch::Tensor out) {
  TORCH_CHECK(kcache.dim() == 3 && kcache.is_contiguous() && vcache.is_contiguous(), "caches [B, Tmax, H*D]");
  TORCH_CHECK(D == 64 || D == 128, "head_dim 64 or 128");
  const int B = (int)kcache.size(0), Tmax = (int)kcache.size(1);
  TORCH_CHECK(kcache.size(2) == H * D && q.stride(-1) == 1 && out.stride(-1) == 1, "layout");
  c10::cuda::CUDAGuard g(q.device());
  const size_t smem = (size_t)Tmax * sizeof(float);
  auto s = at::cuda::getCurrentCUDAStream();
  auto* qp = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  auto* kp = reinterpret_cast<const __nv_bfloat16*>(kcache.data_ptr());
  auto* vp = reinterpret_cast<const __nv_bfloat16*>(vcache.data_ptr());
  auto* op = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (D == 128) {
    if (smem > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(decode_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    decode_attn_kernel<128><<<B * H, kDecThreads, smem, s>>>(qp, q.stride(0), kp, vp, kcache.stride(1), kcache.stride(0),
                                                              len.data_ptr<int>(), Tmax, op, out.stride(0), (int)H, (float)scale);
  } else {
    if (smem > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(decode_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    decode_attn_kernel<64><<<B * H, kDecThreads, smem, s>>>(qp, q.stride(0), kp, vp, kcache.stride(1), kcache.stride(0),
                                                             len.data_ptr<int>(), Tmax, op, out.stride(0), (int)H, (float)scale);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_append(torch::Tensor k, torch::Tensor v, torch::Tensor kcache, torch::Tensor vcache, torch::Tensor pos) {
  const int B = (int)kcache.size(0), C = (int)kcache.size(2);
  TORCH_CHECK(C % 8 == 0 && k.stride(-1) == 1 && v.stride(-1) == 1, "rows");
  c10::cuda::CUDAGuard g(k.device());
  const long long n8 = (long long)B * C / 8;
  kv_append_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()), k.stride(0), reinterpret_cast<const __nv_bfloat16*>(v.data_ptr()),
      v.stride(0), reinterpret_cast<__nv_bfloat16*>(kcache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(vcache.data_ptr()),
      kcache.stride(1), kcache.stride(0), pos.data_ptr<int>(), (int)kcache.size(1), B, C);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void step_advance(torch::Tensor counters) {
  step_advance_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(counters.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void argmax_rows(torch::Tensor logits, int64_t V, torch::Tensor idx_out, c10::optional<torch::Tensor> tokens,
                 torch::Tensor counters, int64_t start) {
  const int B = (int)logits.size(0);
  int* tk = tokens.has_value() ? tokens->data_ptr<int>() : nullptr;
  const long long ldt = tokens.has_value() ? tokens->stride(0) : 0;
  const int max_new = tokens.has_value() ? (int)tokens->size(1) : 0;
  argmax_rows_kernel<<<B, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), logits.stride(0), (int)V, idx_out.data_ptr<int>(), tk,
      ldt, counters.data_ptr<int>(), (int)start, max_new);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Strides (batch, head, token) of a KV cache stored token-major [B, T_max, H*D] or
// head-major [B, H, T_max, D]; `tmax` receives T_max.
void cache_strides(const torch::Tensor& c, int64_t H, int64_t D, long long& sb, long long& sh, long long& st,
                          int& tmax) {
  if (c.dim() == 3) {
    TORCH_CHECK(c.size(2) == H * D && c.stride(2) == 1, "token-major cache [B, T_max, H*D]");
    sb = c.stride(0); st = c.stride(1); sh = D; tmax = (int)c.size(1);
  } else {
    TORCH_CHECK(c.dim() == 4 && c.size(1) == H && c.size(3) == D && c.stride(3) == 1,
                "head-major cache [B, H, T_max, D]");
    sb = c.stride(0); sh = c.stride(1); st = c.stride(2); tmax = (int)c.size(2);
  }
}

// ws: fp32 >= B*H*splits*(D+4), 16-byte aligned; cnt: int32 >= B*H, zero before the
// first call (left zeroed).
void decode_attn_split(torch::Tensor q, torch::Tensor kcache, torch::Tensor vcache, torch::Tensor len, int64_t H,
                       int64_t D, double scale, torch::Tensor out, torch::Tensor ws, torch::Tensor cnt,
                       int64_t splits, bool pdl) {
  TORCH_CHECK(D == 128, "split decode attention supports head_dim 128");
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && kcache.scalar_type() == at::kBFloat16 &&
                  vcache.scalar_type() == at::kBFloat16, "bf16 inputs");
  TORCH_CHECK(kcache.sizes() == vcache.sizes() && kcache.strides() == vcache.strides(), "k / v caches alike");
  long long sb, sh, st;
  int tmax;
  cache_strides(kcache, H, D, sb, sh, st, tmax);
  auto a16 = [](const torch::Tensor& t) { return (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0; };
  TORCH_CHECK((q.stride(0) * 2) % 16 == 0 && (sb * 2) % 16 == 0 && (sh * 2) % 16 == 0 && (st * 2) % 16 == 0 &&
                  (out.stride(0) * 2) % 8 == 0 && out.stride(1) == 1 && q.stride(1) == 1,
              "16-byte aligned q / cache rows (8 bf16 per lane), 8-byte aligned output rows");
  TORCH_CHECK(a16(q) && a16(kcache) && a16(vcache) && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 7) == 0,
              "aligned bases");
  const int64_t B = q.size(0);
  TORCH_CHECK(kcache.size(0) >= B, "cache batch");
  TORCH_CHECK(splits >= 1 && splits <= 64, "splits 1..64");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.numel() >= B * H * splits * (D + 4), "workspace size");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ws.data_ptr()) & 15) == 0, "workspace must be 16-byte aligned");
  TORCH_CHECK(cnt.scalar_type() == at::kInt && cnt.numel() >= B * H, "counter size");
  c10::cuda::CUDAGuard guard(q.device());
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)(B * H * splits), 1, 1);
  cfg.blockDim = dim3(kDecThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, decode_attn_split_kernel<128>,
                                    reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), (long long)q.stride(0),
                                    reinterpret_cast<const __nv_bfloat16*>(kcache.data_ptr()),
                                    reinterpret_cast<const __nv_bfloat16*>(vcache.data_ptr()), sb, sh, st,
                                    (const int*)len.data_ptr<int>(), tmax,
                                    reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (long long)out.stride(0), (int)H,
                                    (float)scale, (int)splits, ws.data_ptr<float>(), cnt.data_ptr<int>()));
}


}  // namespace tfb
