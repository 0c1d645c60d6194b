// Memory-bound fused ops of the GPT block, one pass over HBM each:
//   * parameter-free RMSNorm forward / backward (optionally adding a residual grad),
//   * residual mix  xm = l_r * x + l_0 * x0  fused with RMSNorm, and its backward
//     (dl_r, dl_0 reduced in-kernel; dx0 accumulated in fp32 across layers),
//   * embedding gather fused with RMSNorm, and its scatter-add backward,
//   * RoPE + per-head RMSNorm of q and k (QK-norm), forward / backward, in place on
//     the fused [tokens, q|k|v] projection buffer,
//   * softcap S*tanh(z/S) + cross-entropy forward AND backward in one pass over the
//     bf16 logits (the per-row gradient overwrites the logits in place).
// Rows are processed one warp per row with 16-byte vector loads; eps = FLT_EPSILON as
// in F.rms_norm with fp32 opmath.
// Reference counterparts: norm (train.py:1432-1433), RoPE + QK-norm (train.py:1543-1702),
// softcapped cross-entropy (train.py:1768-1925), the embedding lookup and residual mix of
// GPT.forward / Block (train.py:3412-3485, train.py:2631-2764).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

constexpr float kNormEps = 1.1920928955078125e-07f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* f) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* f) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) w[j] = pack_bf16x2(f[2 * j], f[2 * j + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void load8f(const float* p, float* f) {
  float4 a = reinterpret_cast<const float4*>(p)[0];
  float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ void store8f(float* p, const float* f) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// ============================================================================ RMSNorm
// NCH = number of 256-element chunks a warp covers (C <= NCH * 256, C % 8 == 0).
template <int NCH>
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, __nv_bfloat16* __restrict__ y,
                                   long long ldy, float* __restrict__ rstd, int M, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      load8(x + row * ldx + col, v[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[c][j] * v[c][j];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(C) + kNormEps);
  if (lane == 0 && rstd) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * r;
      store8(y + row * ldy + col, o);
    }
  }
}

// dx = r * (dy - xhat * mean(dy * xhat)) (+ dadd), xhat = x * r
template <int NCH>
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, long long lddy,
                                   const __nv_bfloat16* __restrict__ x, long long ldx, const float* __restrict__ rstd,
                                   const __nv_bfloat16* __restrict__ dadd, long long ldadd, __nv_bfloat16* __restrict__ dx,
                                   long long lddx, int M, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float r = rstd[row];
  float g[NCH][8], xh[NCH][8];
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      load8(dy + row * lddy + col, g[c]);
      load8(x + row * ldx + col, xh[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[c][j] *= r;
        dot += g[c][j] * xh[c][j];
      }
    }
  }
  dot = warp_sum(dot) / float(C);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float o[8], a[8];
      if (dadd) load8(dadd + row * ldadd + col, a);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = r * (g[c][j] - xh[c][j] * dot) + (dadd ? a[j] : 0.f);
      store8(dx + row * lddx + col, o);
    }
  }
}

// ============================================================================ mix + norm
// xm = lr * x + l0 * x0 ; h = norm(xm)
template <int NCH>
__global__ void mix_norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ x0,
                                    const float* __restrict__ lam_r, const float* __restrict__ lam_0,
                                    __nv_bfloat16* __restrict__ xm, __nv_bfloat16* __restrict__ h,
                                    float* __restrict__ rstd, int M, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float lr = *lam_r, l0 = *lam_0;
  float v[NCH][8];
  float ss = 0.f;
  const long long base = (long long)row * C;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float a[8], b[8];
      load8(x + base + col, a);
      load8(x0 + base + col, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        // the residual stream is stored in bf16: normalise the rounded value
        v[c][j] = __bfloat162float(__float2bfloat16_rn(lr * a[j] + l0 * b[j]));
        ss += v[c][j] * v[c][j];
      }
      store8(xm + base + col, v[c]);
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(C) + kNormEps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * r;
      store8(h + base + col, o);
    }
  }
}

// g = dxm + norm_bwd(dh); dx = lr * g; dx0_acc (fp32) += l0 * g; dlr += sum(x*g); dl0 += sum(x0*g)
template <int NCH>
__global__ void mix_norm_bwd_kernel(const __nv_bfloat16* __restrict__ dxm, const __nv_bfloat16* __restrict__ dh,
                                    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ x0,
                                    const __nv_bfloat16* __restrict__ xm, const float* __restrict__ rstd,
                                    const float* __restrict__ lam_r, const float* __restrict__ lam_0,
                                    __nv_bfloat16* __restrict__ dx, float* __restrict__ dx0_acc, int dx0_init,
                                    float* __restrict__ dlam_r, float* __restrict__ dlam_0, int M, int C) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  __shared__ float red[2][32];
  float pr = 0.f, p0 = 0.f;
  if (row < M) {
    const float r = rstd[row];
    const float lr = *lam_r, l0 = *lam_0;
    const long long base = (long long)row * C;
    float g[NCH][8], xh[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < C) {
        load8(dh + base + col, g[c]);
        load8(xm + base + col, xh[c]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[c][j] *= r;
          dot += g[c][j] * xh[c][j];
        }
      }
    }
    dot = warp_sum(dot) / float(C);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
      if (col < C) {
        float a[8], xv[8], x0v[8], o[8], acc[8];
        load8(dxm + base + col, a);
        load8(x + base + col, xv);
        load8(x0 + base + col, x0v);
        if (!dx0_init) load8f(dx0_acc + base + col, acc);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float gt = a[j] + r * (g[c][j] - xh[c][j] * dot);
          o[j] = lr * gt;
          acc[j] = (dx0_init ? 0.f : acc[j]) + l0 * gt;
          pr += xv[j] * gt;
          p0 += x0v[j] * gt;
        }
        store8(dx + base + col, o);
        store8f(dx0_acc + base + col, acc);
      }
    }
  }
  pr = warp_sum(pr);
  p0 = warp_sum(p0);
  if (lane == 0) {
    red[0][threadIdx.x >> 5] = pr;
    red[1][threadIdx.x >> 5] = p0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float a = 0.f, b = 0.f;
    for (int w = 0; w < warps; ++w) {
      a += red[0][w];
      b += red[1][w];
    }
    atomicAdd(dlam_r, a);
    atomicAdd(dlam_0, b);
  }
}

// ============================================================================ embed + norm
template <int NCH>
__global__ void embed_norm_fwd_kernel(const int* __restrict__ idx, long long idx_ld, int T,
                                      const float* __restrict__ wte, __nv_bfloat16* __restrict__ out,
                                      float* __restrict__ rstd, int M, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int tok = idx[(long long)(row / T) * idx_ld + (row % T)];
  const float* src = wte + (long long)tok * C;
  float v[NCH][8];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      load8f(src + col, v[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[c][j] = __bfloat162float(__float2bfloat16_rn(v[c][j]));  // .to(bf16) before norm
        ss += v[c][j] * v[c][j];
      }
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(C) + kNormEps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[c][j] * r;
      store8(out + (long long)row * C + col, o);
    }
  }
}

// dwte[tok] += norm_bwd(g) with g = dx0_acc (fp32) (+ dx0 bf16)
template <int NCH>
__global__ void embed_norm_bwd_kernel(const int* __restrict__ idx, long long idx_ld, int T,
                                      const float* __restrict__ wte, const float* __restrict__ rstd,
                                      const float* __restrict__ gacc, const __nv_bfloat16* __restrict__ gb,
                                      float* __restrict__ dwte, int M, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int tok = idx[(long long)(row / T) * idx_ld + (row % T)];
  const float r = rstd[row];
  const float* src = wte + (long long)tok * C;
  float g[NCH][8], xh[NCH][8];
  float dot = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float t[8];
      if (gacc) load8f(gacc + (long long)row * C + col, g[c]);
      else {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[c][j] = 0.f;
      }
      if (gb) {
        load8(gb + (long long)row * C + col, t);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[c][j] += t[j];
      }
      load8f(src + col, xh[c]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xh[c][j] = __bfloat162float(__float2bfloat16_rn(xh[c][j])) * r;
        dot += g[c][j] * xh[c][j];
      }
    }
  }
  dot = warp_sum(dot) / float(C);
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
    if (col < C) {
      float* dst = dwte + (long long)tok * C + col;
#pragma unroll
      for (int j = 0; j < 8; j += 4)
        atomicAdd(reinterpret_cast<float4*>(dst + j),
                  make_float4(r * (g[c][j] - xh[c][j] * dot), r * (g[c][j + 1] - xh[c][j + 1] * dot),
                              r * (g[c][j + 2] - xh[c][j + 2] * dot), r * (g[c][j + 3] - xh[c][j + 3] * dot)));
    }
  }
}

// ============================================================================ RoPE + QK-norm
// One warp per (token, head).  Head vectors of D = 64 or 128 (D/2 rotation pairs);
// lane l owns pairs [l*P, l*P+P) with P = D/64 ... generalised as "pairs per lane".
// y1 = x1 cos + x2 sin ; y2 = -x1 sin + x2 cos ; z = y * rsqrt(mean(y^2) + eps)
template <int PPL>  // pairs per lane: D = 64 * PPL
__global__ void rope_norm_fwd_kernel(__nv_bfloat16* __restrict__ buf, long long ld_tok, int head0, int nheads,
                                     const __nv_bfloat16* __restrict__ cosb, const __nv_bfloat16* __restrict__ sinb,
                                     int T, int pos_offset, float* __restrict__ rstd, int M,
                                     __nv_bfloat16* __restrict__ out, long long ld_out, const int* __restrict__ pos_ptr) {
  constexpr int D = 64 * PPL, HALF = D / 2;
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long long)M * nheads) return;
  const int row = (int)(w / nheads), hh = (int)(w % nheads);
  const int pos = row % T + (pos_ptr ? *pos_ptr : pos_offset);
  __nv_bfloat16* src = buf + (long long)row * ld_tok + (long long)(head0 + hh) * D;
  __nv_bfloat16* dst = out ? out + (long long)row * ld_out + (long long)(head0 + hh) * D : src;
  float y1[PPL], y2[PPL];
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    const int i = lane * PPL + p;
    const float x1 = __bfloat162float(src[i]), x2 = __bfloat162float(src[i + HALF]);
    const float c = __bfloat162float(cosb[(long long)pos * HALF + i]);
    const float s = __bfloat162float(sinb[(long long)pos * HALF + i]);
    y1[p] = x1 * c + x2 * s;
    y2[p] = x2 * c - x1 * s;
    ss += y1[p] * y1[p] + y2[p] * y2[p];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / float(D) + kNormEps);
  if (lane == 0 && rstd) rstd[w] = r;
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    const int i = lane * PPL + p;
    dst[i] = __float2bfloat16_rn(y1[p] * r);
    dst[i + HALF] = __float2bfloat16_rn(y2[p] * r);
  }
}

// In place on the gradient buffer: dy = r (g - z mean(g z)); dx = rope^T(dy)
template <int PPL>
__global__ void rope_norm_bwd_kernel(__nv_bfloat16* __restrict__ gbuf, long long ld_g, const __nv_bfloat16* __restrict__ zbuf,
                                     long long ld_z, int head0, int nheads, const __nv_bfloat16* __restrict__ cosb,
                                     const __nv_bfloat16* __restrict__ sinb, int T, const float* __restrict__ rstd, int M) {
  constexpr int D = 64 * PPL, HALF = D / 2;
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long long)M * nheads) return;
  const int row = (int)(w / nheads), hh = (int)(w % nheads);
  const int pos = row % T;
  __nv_bfloat16* g = gbuf + (long long)row * ld_g + (long long)(head0 + hh) * D;
  const __nv_bfloat16* z = zbuf + (long long)row * ld_z + (long long)(head0 + hh) * D;
  const float r = rstd[w];
  float g1[PPL], g2[PPL], z1[PPL], z2[PPL];
  float dot = 0.f;
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    const int i = lane * PPL + p;
    g1[p] = __bfloat162float(g[i]);
    g2[p] = __bfloat162float(g[i + HALF]);
    z1[p] = __bfloat162float(z[i]);
    z2[p] = __bfloat162float(z[i + HALF]);
    dot += g1[p] * z1[p] + g2[p] * z2[p];
  }
  dot = warp_sum(dot) / float(D);
#pragma unroll
  for (int p = 0; p < PPL; ++p) {
    const int i = lane * PPL + p;
    const float d1 = r * (g1[p] - z1[p] * dot), d2 = r * (g2[p] - z2[p] * dot);
    const float c = __bfloat162float(cosb[(long long)pos * HALF + i]);
    const float s = __bfloat162float(sinb[(long long)pos * HALF + i]);
    // transpose of [[c, s], [-s, c]] applied to (d1, d2)
    g[i] = __float2bfloat16_rn(d1 * c - d2 * s);
    g[i + HALF] = __float2bfloat16_rn(d1 * s + d2 * c);
  }
}

// ============================================================================ softcap CE
// One CTA (256 threads) per row of bf16 logits z[V_pad]; only the first V columns are
// real classes.  y = S tanh(z / S); loss = log sum_j exp(y_j) - y_c, computed with the
// fixed shift S (|y| < S, so exp(y - S) never overflows and the sum stays >= exp(-2S)).
// In the same pass the gradient w.r.t. z is written over the logits:
//   dz_j = w_row * scale * (softmax(y)_j - [j == c]) * (1 - t_j^2);  padded columns 0.
template <typename TT>
__global__ void softcap_ce_kernel(__nv_bfloat16* __restrict__ logits, long long ld, const TT* __restrict__ tgt,
                                  long long tgt_ld, int T, const float* __restrict__ row_w, int V, int Vpad,
                                  float S, float scale, float* __restrict__ loss_out, int write_grad) {
  const int row = blockIdx.x;
  const int b = row / T, t = row % T;
  const long long c_ll = (long long)tgt[(long long)b * tgt_ld + t];
  __nv_bfloat16* z = logits + (long long)row * ld;
  __shared__ float red[32];
  const int tid = threadIdx.x, nt = blockDim.x;
  const float invS = 1.f / S;
  const bool valid = c_ll >= 0 && c_ll < V;
  // The target's capped logit, read by the thread that writes the loss before any
  // thread can reach the gradient pass (which overwrites the row after two barriers).
  float yc = 0.f;
  if (tid == 0 && valid) yc = S * tanhf(__bfloat162float(z[c_ll]) * invS);
  float sum = 0.f;
  for (int j0 = tid * 8; j0 < Vpad; j0 += nt * 8) {
    float f[8];
    load8(z + j0, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = j0 + k;
      if (j < V) sum += __expf(S * tanhf(f[k] * invS) - S);
    }
  }
  sum = warp_sum(sum);
  if ((tid & 31) == 0) red[tid >> 5] = sum;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (nt >> 5) ? red[tid] : 0.f;
    v = warp_sum(v);
    if (tid == 0) red[0] = v;
  }
  __syncthreads();
  const float total = red[0];
  const float w = valid ? (row_w ? row_w[row] : 1.f) : 0.f;
  if (tid == 0) loss_out[row] = valid ? w * (S + logf(total) - yc) : 0.f;
  if (!write_grad) return;
  const float inv_total = 1.f / total;
  const float gs = w * scale;
  for (int j0 = tid * 8; j0 < Vpad; j0 += nt * 8) {
    float f[8], o[8];
    load8(z + j0, f);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = j0 + k;
      if (j < V && gs != 0.f) {
        const float th = tanhf(f[k] * invS);
        const float p = __expf(S * th - S) * inv_total;
        o[k] = gs * (p - (j == c_ll ? 1.f : 0.f)) * (1.f - th * th);
      } else {
        o[k] = 0.f;
      }
    }
    store8(z + j0, o);
  }
}

// ============================================================================ host wrappers
static inline int nch_for(int C) { return (C + 255) / 256; }

#define TFB_NCH_DISPATCH(C, ...)                                                   \
  switch (nch_for(C)) {                                                            \
    case 1: { constexpr int NCH = 1; __VA_ARGS__; break; }                         \
    case 2: { constexpr int NCH = 2; __VA_ARGS__; break; }                         \
    case 3: { constexpr int NCH = 3; __VA_ARGS__; break; }                         \
    case 4: { constexpr int NCH = 4; __VA_ARGS__; break; }                         \
    case 5: { constexpr int NCH = 5; __VA_ARGS__; break; }                         \
    case 6: { constexpr int NCH = 6; __VA_ARGS__; break; }                         \
    case 7: { constexpr int NCH = 7; __VA_ARGS__; break; }                         \
    case 8: { constexpr int NCH = 8; __VA_ARGS__; break; }                         \
    default: TORCH_CHECK(false, "row width ", C, " exceeds 2048");                 \
  }

static void check_bf16_rows(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, name, " must be a CUDA bf16 tensor");
  TORCH_CHECK(t.stride(-1) == 1, name, " must have a contiguous last dimension");
}

void rmsnorm_fwd(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> rstd) {
  check_bf16_rows(x, "x");
  check_bf16_rows(y, "y");
  const int C = (int)x.size(-1);
  const int M = (int)(x.numel() / C);
  TORCH_CHECK(C % 8 == 0, "C % 8");
  c10::cuda::CUDAGuard g(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const long long ldx = x.dim() >= 2 ? x.stride(-2) : C, ldy = y.dim() >= 2 ? y.stride(-2) : C;
  float* r = rstd.has_value() ? rstd->data_ptr<float>() : nullptr;
  const int wpb = 8;
  dim3 grid((M + wpb - 1) / wpb);
  TFB_NCH_DISPATCH(C, rmsnorm_fwd_kernel<NCH><<<grid, wpb * 32, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), ldx, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), ldy, r, M, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rmsnorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor rstd, c10::optional<torch::Tensor> dadd,
                 torch::Tensor dx) {
  check_bf16_rows(dy, "dy");
  check_bf16_rows(x, "x");
  check_bf16_rows(dx, "dx");
  const int C = (int)x.size(-1);
  const int M = (int)(x.numel() / C);
  c10::cuda::CUDAGuard g(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const __nv_bfloat16* da = dadd.has_value() ? reinterpret_cast<const __nv_bfloat16*>(dadd->data_ptr()) : nullptr;
  const long long lda = dadd.has_value() ? dadd->stride(-2) : 0;
  const int wpb = 8;
  dim3 grid((M + wpb - 1) / wpb);
  TFB_NCH_DISPATCH(C, rmsnorm_bwd_kernel<NCH><<<grid, wpb * 32, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), dy.stride(-2), reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()),
      x.stride(-2), rstd.data_ptr<float>(), da, lda, reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx.stride(-2), M, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mix_norm_fwd(torch::Tensor x, torch::Tensor x0, torch::Tensor lr, torch::Tensor l0, torch::Tensor xm,
                  torch::Tensor h, torch::Tensor rstd) {
  for (auto* t : {&x, &x0, &xm, &h}) TORCH_CHECK(t->is_contiguous() && t->scalar_type() == at::kBFloat16, "bf16 contiguous");
  const int C = (int)x.size(-1);
  const int M = (int)(x.numel() / C);
  c10::cuda::CUDAGuard g(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int wpb = 8;
  dim3 grid((M + wpb - 1) / wpb);
  TFB_NCH_DISPATCH(C, mix_norm_fwd_kernel<NCH><<<grid, wpb * 32, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x0.data_ptr()),
      lr.data_ptr<float>(), l0.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(xm.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), rstd.data_ptr<float>(), M, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void mix_norm_bwd(torch::Tensor dxm, torch::Tensor dh, torch::Tensor x, torch::Tensor x0, torch::Tensor xm,
                  torch::Tensor rstd, torch::Tensor lr, torch::Tensor l0, torch::Tensor dx, torch::Tensor dx0_acc,
                  bool dx0_init, torch::Tensor dlr, torch::Tensor dl0) {
  for (auto* t : {&dxm, &dh, &x, &x0, &xm, &dx}) TORCH_CHECK(t->is_contiguous() && t->scalar_type() == at::kBFloat16, "bf16 contiguous");
  TORCH_CHECK(dx0_acc.is_contiguous() && dx0_acc.scalar_type() == at::kFloat, "dx0_acc fp32");
  const int C = (int)x.size(-1);
  const int M = (int)(x.numel() / C);
  c10::cuda::CUDAGuard g(x.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int wpb = 8;
  dim3 grid((M + wpb - 1) / wpb);
  TFB_NCH_DISPATCH(C, mix_norm_bwd_kernel<NCH><<<grid, wpb * 32, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(dxm.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(x0.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(xm.data_ptr()), rstd.data_ptr<float>(), lr.data_ptr<float>(),
      l0.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), dx0_acc.data_ptr<float>(), dx0_init ? 1 : 0,
      dlr.data_ptr<float>(), dl0.data_ptr<float>(), M, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_norm_fwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor out, torch::Tensor rstd) {
  TORCH_CHECK(idx.scalar_type() == at::kInt && idx.dim() == 2 && idx.stride(1) == 1, "idx int32 [B,T]");
  TORCH_CHECK(wte.scalar_type() == at::kFloat && wte.is_contiguous(), "wte fp32");
  const int C = (int)wte.size(1);
  const int T = (int)idx.size(1);
  const int M = (int)(idx.size(0) * T);
  c10::cuda::CUDAGuard g(wte.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int wpb = 8;
  dim3 grid((M + wpb - 1) / wpb);
  TFB_NCH_DISPATCH(C, embed_norm_fwd_kernel<NCH><<<grid, wpb * 32, 0, s>>>(
      idx.data_ptr<int>(), idx.stride(0), T, wte.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      rstd.data_ptr<float>(), M, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void embed_norm_bwd(torch::Tensor idx, torch::Tensor wte, torch::Tensor rstd, c10::optional<torch::Tensor> gacc,
                    c10::optional<torch::Tensor> gb, torch::Tensor dwte) {
  const int C = (int)wte.size(1);
  const int T = (int)idx.size(1);
  const int M = (int)(idx.size(0) * T);
  TORCH_CHECK(dwte.scalar_type() == at::kFloat && dwte.is_contiguous(), "dwte fp32");
  c10::cuda::CUDAGuard g(wte.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int wpb = 8;
  dim3 grid((M + wpb - 1) / wpb);
  const float* ga = gacc.has_value() ? gacc->data_ptr<float>() : nullptr;
  const __nv_bfloat16* gbp = gb.has_value() ? reinterpret_cast<const __nv_bfloat16*>(gb->data_ptr()) : nullptr;
  TFB_NCH_DISPATCH(C, embed_norm_bwd_kernel<NCH><<<grid, wpb * 32, 0, s>>>(
      idx.data_ptr<int>(), idx.stride(0), T, wte.data_ptr<float>(), rstd.data_ptr<float>(), ga, gbp,
      dwte.data_ptr<float>(), M, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// buf: [M, ld_tok] bf16, heads [head0, head0+nheads) of width D are rotated+normed.
void rope_norm_fwd(torch::Tensor buf, int64_t head0, int64_t nheads, int64_t D, torch::Tensor cos,
                   torch::Tensor sin, int64_t T, int64_t pos_offset, c10::optional<torch::Tensor> rstd,
                   c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> pos_t) {
  check_bf16_rows(buf, "buf");
  TORCH_CHECK(cos.is_contiguous() && sin.is_contiguous() && cos.scalar_type() == at::kBFloat16, "cos/sin bf16");
  const long long ld = buf.stride(-2);
  const int M = (int)(buf.numel() / buf.size(-1));
  c10::cuda::CUDAGuard g(buf.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const long long warps = (long long)M * nheads;
  const int wpb = 8;
  dim3 grid((unsigned)((warps + wpb - 1) / wpb));
  float* r = rstd.has_value() ? rstd->data_ptr<float>() : nullptr;
  __nv_bfloat16* o = out.has_value() ? reinterpret_cast<__nv_bfloat16*>(out->data_ptr()) : nullptr;
  const long long ldo = out.has_value() ? out->stride(-2) : 0;
  auto* b = reinterpret_cast<__nv_bfloat16*>(buf.data_ptr());
  auto* cp = reinterpret_cast<const __nv_bfloat16*>(cos.data_ptr());
  auto* sp = reinterpret_cast<const __nv_bfloat16*>(sin.data_ptr());
  const int* pp = pos_t.has_value() ? pos_t->data_ptr<int>() : nullptr;
  if (D == 128) rope_norm_fwd_kernel<2><<<grid, wpb * 32, 0, s>>>(b, ld, (int)head0, (int)nheads, cp, sp, (int)T, (int)pos_offset, r, M, o, ldo, pp);
  else if (D == 64) rope_norm_fwd_kernel<1><<<grid, wpb * 32, 0, s>>>(b, ld, (int)head0, (int)nheads, cp, sp, (int)T, (int)pos_offset, r, M, o, ldo, pp);
  else if (D == 256) rope_norm_fwd_kernel<4><<<grid, wpb * 32, 0, s>>>(b, ld, (int)head0, (int)nheads, cp, sp, (int)T, (int)pos_offset, r, M, o, ldo, pp);
  else TORCH_CHECK(false, "head_dim must be 64, 128 or 256");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void rope_norm_bwd(torch::Tensor gbuf, torch::Tensor zbuf, int64_t head0, int64_t nheads, int64_t D,
                   torch::Tensor cos, torch::Tensor sin, int64_t T, torch::Tensor rstd) {
  check_bf16_rows(gbuf, "gbuf");
  check_bf16_rows(zbuf, "zbuf");
  const int M = (int)(gbuf.numel() / gbuf.size(-1));
  c10::cuda::CUDAGuard g(gbuf.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const long long warps = (long long)M * nheads;
  const int wpb = 8;
  dim3 grid((unsigned)((warps + wpb - 1) / wpb));
  auto* gp = reinterpret_cast<__nv_bfloat16*>(gbuf.data_ptr());
  auto* zp = reinterpret_cast<const __nv_bfloat16*>(zbuf.data_ptr());
  auto* cp = reinterpret_cast<const __nv_bfloat16*>(cos.data_ptr());
  auto* sp = reinterpret_cast<const __nv_bfloat16*>(sin.data_ptr());
  const long long ldg = gbuf.stride(-2), ldz = zbuf.stride(-2);
  if (D == 128) rope_norm_bwd_kernel<2><<<grid, wpb * 32, 0, s>>>(gp, ldg, zp, ldz, (int)head0, (int)nheads, cp, sp, (int)T, rstd.data_ptr<float>(), M);
  else if (D == 64) rope_norm_bwd_kernel<1><<<grid, wpb * 32, 0, s>>>(gp, ldg, zp, ldz, (int)head0, (int)nheads, cp, sp, (int)T, rstd.data_ptr<float>(), M);
  else if (D == 256) rope_norm_bwd_kernel<4><<<grid, wpb * 32, 0, s>>>(gp, ldg, zp, ldz, (int)head0, (int)nheads, cp, sp, (int)T, rstd.data_ptr<float>(), M);
  else TORCH_CHECK(false, "head_dim must be 64, 128 or 256");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// logits: [N, Vpad] bf16 rows (ld = row stride); targets [B, T] (any int type, row stride
// tgt_ld); returns per-row loss (fp32) and, if write_grad, overwrites logits with dL/dz.
void softcap_ce(torch::Tensor logits, torch::Tensor targets, int64_t T, c10::optional<torch::Tensor> row_w,
                int64_t V, double S, double scale, torch::Tensor loss, bool write_grad) {
  check_bf16_rows(logits, "logits");
  const int N = (int)logits.size(0);
  const int Vpad = (int)logits.size(1);
  TORCH_CHECK(Vpad % 8 == 0 && V <= Vpad, "vocab padding");
  TORCH_CHECK(loss.scalar_type() == at::kFloat && loss.numel() >= N, "loss fp32 [N]");
  TORCH_CHECK(targets.dim() == 2 && targets.stride(1) == 1, "targets [B, T] with unit inner stride");
  c10::cuda::CUDAGuard g(logits.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const float* w = row_w.has_value() ? row_w->data_ptr<float>() : nullptr;
  auto* z = reinterpret_cast<__nv_bfloat16*>(logits.data_ptr());
  if (targets.scalar_type() == at::kLong)
    softcap_ce_kernel<int64_t><<<N, 256, 0, s>>>(z, logits.stride(0), targets.data_ptr<int64_t>(), targets.stride(0), (int)T, w,
                                                  (int)V, Vpad, (float)S, (float)scale, loss.data_ptr<float>(), write_grad ? 1 : 0);
  else if (targets.scalar_type() == at::kInt)
    softcap_ce_kernel<int32_t><<<N, 256, 0, s>>>(z, logits.stride(0), targets.data_ptr<int32_t>(), targets.stride(0), (int)T, w,
                                                  (int)V, Vpad, (float)S, (float)scale, loss.data_ptr<float>(), write_grad ? 1 : 0);
  else TORCH_CHECK(false, "targets must be int32 or int64");
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tfb
