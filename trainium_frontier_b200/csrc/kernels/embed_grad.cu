// Deterministic embedding gradient: dwte[v] += sum over the positions t with idx[t] == v of
// norm_bwd(g[t]) (g = the fp32 x0 accumulator (+ the bf16 gradient of the normed
// embedding), norm_bwd the parameter-free RMSNorm backward at the token's bf16 row), summed
// in position order, so the result is bitwise the same from run to run.
//
//   1. per block of 1024 positions, a token histogram (shared-memory counts);
//   2. per token, the block-by-block prefix of those counts and the token's total;
//   3. one block: the exclusive scan of the totals (segment starts) and of the tokens'
//      chunk counts (work items of at most kEgChunk positions);
//   4. per block of positions, a stable placement: positions in order, one warp, each
//      position's rank among the earlier same-token positions of its block from
//      __match_any_sync plus running shared-memory counts -- perm[] lists every token's
//      positions in increasing order;
//   5. one CTA per work item (token v, chunk c): eight warps take the chunk's positions
//      round-robin, each accumulating norm_bwd rows in registers, and the eight partial
//      rows are added in warp order; a token of one chunk adds straight into dwte[v], a
//      longer one writes its chunk partials;
//   6. per token with several chunks, the partials are added in chunk order into dwte[v].
//
// Reference counterpart: the embedding gradient of GPT.forward's wte lookup and norm
// (train.py:3416, :3433), whose CUDA index-add accumulates in a data-dependent order.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

namespace {

constexpr int kEgBlock = 1024;  // positions per histogram / placement block
constexpr int kEgChunk = 256;   // positions per work item
constexpr int kEgMaxV = 8192;   // vocabulary bound of the shared-memory histogram (32 KB)

__global__ void eg_hist_kernel(const int* __restrict__ idx, long long idx_ld, int T, int M, int V,
                               int* __restrict__ cnt /* [G][V] */) {
  __shared__ int h[kEgMaxV];
  for (int v = threadIdx.x; v < V; v += blockDim.x) h[v] = 0;
  __syncthreads();
  const int p = blockIdx.x * kEgBlock + threadIdx.x;
  if (p < M) atomicAdd(&h[idx[(long long)(p / T) * idx_ld + p % T]], 1);
  __syncthreads();
  for (int v = threadIdx.x; v < V; v += blockDim.x) cnt[(long long)blockIdx.x * V + v] = h[v];
}

// per token: off[g][v] = sum_{g' < g} cnt[g'][v]; total[v]
__global__ void eg_colscan_kernel(int* __restrict__ cnt, int G, int V, int* __restrict__ total) {
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= V) return;
  int run = 0;
  for (int g = 0; g < G; ++g) {
    const int c = cnt[(long long)g * V + v];
    cnt[(long long)g * V + v] = run;
    run += c;
  }
  total[v] = run;
}

// one block: start[v] = exclusive scan of total; item0[v] = exclusive scan of ceil(total / chunk);
// item0[V] = number of work items
__global__ void eg_scan_kernel(const int* __restrict__ total, int V, int* __restrict__ start, int* __restrict__ item0) {
  __shared__ int ps[1024], pi[1024];
  const int per = (V + 1023) / 1024;
  const int v0 = threadIdx.x * per;
  int s = 0, it = 0;
  for (int v = v0; v < min(V, v0 + per); ++v) {
    s += total[v];
    it += (total[v] + kEgChunk - 1) / kEgChunk;
  }
  ps[threadIdx.x] = s;
  pi[threadIdx.x] = it;
  __syncthreads();
  if (threadIdx.x == 0) {  // 1024 partial sums in order
    int a = 0, b = 0;
    for (int t = 0; t < 1024; ++t) {
      const int x = ps[t], y = pi[t];
      ps[t] = a;
      pi[t] = b;
      a += x;
      b += y;
    }
    item0[V] = b;
  }
  __syncthreads();
  s = ps[threadIdx.x];
  it = pi[threadIdx.x];
  for (int v = v0; v < min(V, v0 + per); ++v) {
    start[v] = s;
    item0[v] = it;
    s += total[v];
    it += (total[v] + kEgChunk - 1) / kEgChunk;
  }
}

// one warp per block of positions, positions in order
__global__ void eg_place_kernel(const int* __restrict__ idx, long long idx_ld, int T, int M, int V,
                                const int* __restrict__ off /* [G][V] */, const int* __restrict__ start,
                                int* __restrict__ perm) {
  __shared__ int run[kEgMaxV];
  const int lane = threadIdx.x;
  for (int v = lane; v < V; v += 32) run[v] = 0;
  __syncwarp();
  const int g = blockIdx.x;
  for (int base = g * kEgBlock; base < min(M, (g + 1) * kEgBlock); base += 32) {
    const int p = base + lane;
    const bool in = p < M;
    const int v = in ? idx[(long long)(p / T) * idx_ld + p % T] : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffffu, v);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    int prior = 0;
    if (in) prior = run[v];
    __syncwarp();
    if (in) {
      perm[start[v] + off[(long long)g * V + v] + prior + rank] = p;
      if (rank == 0) run[v] = prior + __popc(peers);
    }
    __syncwarp();
  }
}

// one CTA (8 warps) per work item; C <= 2048 (64 fp32 per lane)
template <int NCH>
__global__ void eg_accum_kernel(const int* __restrict__ perm, const int* __restrict__ start, const int* __restrict__ total,
                                const int* __restrict__ item0, int V, const float* __restrict__ wte,
                                const float* __restrict__ rstd, const float* __restrict__ gacc,
                                const __nv_bfloat16* __restrict__ gb, int C, float* __restrict__ dwte,
                                float* __restrict__ part) {
  const int b = blockIdx.x;
  if (b >= item0[V]) return;
  int lo = 0, hi = V - 1;  // last v with item0[v] <= b
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (item0[mid] <= b) lo = mid;
    else hi = mid - 1;
  }
  const int v = lo;
  const int chunk = b - item0[v];
  const int n_chunks = (total[v] + kEgChunk - 1) / kEgChunk;
  const int p0 = start[v] + chunk * kEgChunk;
  const int p1 = start[v] + min(total[v], (chunk + 1) * kEgChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the token's bf16 row, shared by every position
  float xb[NCH][8], acc[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = c * 256 + lane * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc[c][j] = 0.f;
      xb[c][j] = (col + j < C) ? __bfloat162float(__float2bfloat16_rn(wte[(long long)v * C + col + j])) : 0.f;
    }
  }
  for (int q = p0 + warp; q < p1; q += 8) {
    const int row = perm[q];
    const float r = rstd[row];
    float g[NCH][8];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const int col = c * 256 + lane * 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float gv = 0.f;
        if (col + j < C) {
          if (gacc) gv = gacc[(long long)row * C + col + j];
          if (gb) gv += __bfloat162float(gb[(long long)row * C + col + j]);
        }
        g[c][j] = gv;
        dot += gv * (xb[c][j] * r);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot /= (float)C;
#pragma unroll
    for (int c = 0; c < NCH; ++c)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[c][j] += r * (g[c][j] - xb[c][j] * r * dot);
  }
  // add the eight warps' rows in warp order (dynamic shared memory [8][C])
  extern __shared__ float red[];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = c * 256 + lane * 8 + j;
      if (col < C) red[warp * C + col] = acc[c][j];
    }
  __syncthreads();
  for (int col = threadIdx.x; col < C; col += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w * C + col];
    if (n_chunks == 1) dwte[(long long)v * C + col] += s;
    else part[(long long)b * C + col] = s;
  }
}

// tokens of several chunks: dwte[v] += their partials in chunk order
__global__ void eg_partial_kernel(const int* __restrict__ total, const int* __restrict__ item0, int V, int C,
                                  const float* __restrict__ part, float* __restrict__ dwte) {
  const int v = blockIdx.x;
  const int n = (total[v] + kEgChunk - 1) / kEgChunk;
  if (n <= 1) return;
  for (int col = threadIdx.x; col < C; col += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < n; ++k) s += part[(long long)(item0[v] + k) * C + col];
    dwte[(long long)v * C + col] += s;
  }
}

}  // namespace

// idx int32 [B, T] (unit inner stride); wte fp32 [V, C]; rstd fp32 [B*T]; gacc fp32 [B*T, C]
// or none; gb bf16 [B*T, C] or none; dwte fp32 [V, C] (accumulated).
void embed_grad_det(torch::Tensor idx, torch::Tensor wte, torch::Tensor rstd, c10::optional<torch::Tensor> gacc,
                    c10::optional<torch::Tensor> gb, torch::Tensor dwte) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kInt && idx.dim() == 2 && idx.stride(1) == 1, "idx int32 [B, T]");
  TORCH_CHECK(wte.scalar_type() == at::kFloat && wte.is_contiguous() && wte.dim() == 2, "wte fp32 [V, C]");
  const int V = (int)wte.size(0), C = (int)wte.size(1);
  const int T = (int)idx.size(1), M = (int)(idx.size(0) * T);
  TORCH_CHECK(V <= kEgMaxV && C <= 2048, "vocabulary <= 8192, width <= 2048");
  TORCH_CHECK(dwte.scalar_type() == at::kFloat && dwte.is_contiguous() && dwte.numel() == (long long)V * C, "dwte fp32 like wte");
  if (gacc.has_value()) TORCH_CHECK(gacc->scalar_type() == at::kFloat && gacc->is_contiguous(), "gacc fp32 [M, C]");
  if (gb.has_value()) TORCH_CHECK(gb->scalar_type() == at::kBFloat16 && gb->is_contiguous(), "gb bf16 [M, C]");
  c10::cuda::CUDAGuard guard(idx.device());
  auto s = at::cuda::getCurrentCUDAStream();
  const int G = (M + kEgBlock - 1) / kEgBlock;
  auto opt = idx.options();
  auto cnt = torch::empty({(long long)G * V}, opt);
  auto total = torch::empty({V}, opt);
  auto start = torch::empty({V}, opt);
  auto item0 = torch::empty({V + 1}, opt);
  auto perm = torch::empty({M}, opt);
  const int max_items = V + (M + kEgChunk - 1) / kEgChunk;
  auto part = torch::empty({(long long)max_items * C}, wte.options());
  const int* ip = idx.data_ptr<int>();
  eg_hist_kernel<<<G, kEgBlock, 0, s>>>(ip, idx.stride(0), T, M, V, cnt.data_ptr<int>());
  eg_colscan_kernel<<<(V + 255) / 256, 256, 0, s>>>(cnt.data_ptr<int>(), G, V, total.data_ptr<int>());
  eg_scan_kernel<<<1, 1024, 0, s>>>(total.data_ptr<int>(), V, start.data_ptr<int>(), item0.data_ptr<int>());
  eg_place_kernel<<<G, 32, 0, s>>>(ip, idx.stride(0), T, M, V, cnt.data_ptr<int>(), start.data_ptr<int>(),
                                   perm.data_ptr<int>());
  const float* ga = gacc.has_value() ? gacc->data_ptr<float>() : nullptr;
  const __nv_bfloat16* gbp = gb.has_value() ? reinterpret_cast<const __nv_bfloat16*>(gb->data_ptr()) : nullptr;
  const int nch = (C + 255) / 256;
  const size_t red_bytes = (size_t)8 * C * sizeof(float);
#define TFB_EG(N) \
  C10_CUDA_CHECK(cudaFuncSetAttribute(eg_accum_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)red_bytes)); \
  eg_accum_kernel<N><<<max_items, 256, red_bytes, s>>>(perm.data_ptr<int>(), start.data_ptr<int>(), total.data_ptr<int>(), \
                                               item0.data_ptr<int>(), V, wte.data_ptr<float>(), rstd.data_ptr<float>(), \
                                               ga, gbp, C, dwte.data_ptr<float>(), part.data_ptr<float>())
  switch (nch) {
    case 1: TFB_EG(1); break;
    case 2: TFB_EG(2); break;
    case 3: TFB_EG(3); break;
    case 4: TFB_EG(4); break;
    case 5: TFB_EG(5); break;
    case 6: TFB_EG(6); break;
    case 7: TFB_EG(7); break;
    case 8: TFB_EG(8); break;
    default: TORCH_CHECK(false, "width");
  }
#undef TFB_EG
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  eg_partial_kernel<<<V, 256, 0, s>>>(total.data_ptr<int>(), item0.data_ptr<int>(), V, C, part.data_ptr<float>(),
                                      dwte.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tfb
