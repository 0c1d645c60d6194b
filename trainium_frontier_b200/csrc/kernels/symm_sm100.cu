// Fused NVLink collectives of data-parallel distributed Muon, over symmetric memory.
//
// Every rank's flat gradient buffer and update buffer are symmetric allocations (same
// offsets on every GPU, peer base addresses exchanged once).  Instead of NCCL calls:
//
//   symm_barrier     bounded device-side barrier over NVLink (flag stores with release
//                    semantics into each peer's signal pad, acquire loads of our own pad,
//                    monotonically increasing epochs so pads are never reset);
//   symm_rs          reduce-scatter of one gradient bucket: each rank reads ITS owned
//                    segment from every peer (16-byte P2P loads, or one multimem
//                    ld_reduce through the NVSwitch when the multicast object exists),
//                    averages, writes the fp32 result and accumulates its sum of squares
//                    (the global-norm partial) -- reduce + norm in one pass;
//   muon_pre         clip scale, momentum lerp, Nesterov lerp, bf16 cast and per-matrix
//                    sum of squares (Frobenius norm) of the owner's stacks in one pass
//                    (kMuonPreBlocks partial sums per matrix, added in order later);
//   symm_ag_apply    all-gather + apply: for every matrix of a bucket, read its bf16
//                    update from the owner's update buffer (peer load) and apply
//                    w -= bf16(lr) g + lr wd w [g w >= 0] to the fp32 master and its bf16
//                    cache in the same pass.
// Every wait is bounded (2 s) and reports into the device error word; the peer loads
// are plain ld.global (no TMA, no cluster broadcast).
// Reference counterparts: sync_gradients (train.py:4412-4420), the Muon math
// (train.py:3540-3647) and its update kernel (train.py:2023-2078).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

constexpr int kMaxRanks = 8;
constexpr int kMuonPreBlocks = 64;  // blocks (and partial sums) per matrix of muon_pre

struct PeerF32 { const float* p[kMaxRanks]; };
struct PeerBf16 { const __nv_bfloat16* p[kMaxRanks]; };
struct PeerU32 { uint32_t* p[kMaxRanks]; };

__device__ __forceinline__ void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// ------------------------------------------------------------------------------ barrier
// pads.p[r] = rank r's signal pad; slot s of a pad is written by rank s.
__global__ void symm_barrier_kernel(PeerU32 pads, int rank, int world, uint32_t epoch, int* err) {
  const int t = threadIdx.x;
  if (t < world) {
    __threadfence_system();
    st_release_sys(pads.p[t] + rank, epoch);
  }
  __syncthreads();
  if (t < world) {
    const uint32_t* mine = pads.p[rank] + t;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
      const uint32_t v = ld_acquire_sys(mine);
      if ((int)(v - epoch) >= 0) break;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        atomicOr(err, ERR_TIMEOUT_PEER);
        break;
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------ reduce-scatter
// out[i] = inv * sum_r peers[r][src_off + i], i < n (n % 4 == 0); sumsq += sum out^2.
__global__ void symm_rs_kernel(PeerF32 peers, int world, long long src_off, long long n, float* __restrict__ out,
                               float inv, float* __restrict__ sumsq, const float* __restrict__ mc_base) {
  float ss = 0.f;
  const long long n4 = n >> 2;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < n4; v += (long long)gridDim.x * blockDim.x) {
    float4 acc;
    if (mc_base) {
      const float* addr = mc_base + src_off + v * 4;
      asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(acc.x), "=f"(acc.y), "=f"(acc.z), "=f"(acc.w)
                   : "l"(addr)
                   : "memory");
    } else {
      acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int r = 0; r < world; ++r) {
        const float4 x = reinterpret_cast<const float4*>(peers.p[r] + src_off)[v];
        acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
      }
    }
    acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
    reinterpret_cast<float4*>(out)[v] = acc;
    ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    if (sumsq) atomicAdd(sumsq, t);
  }
}

// ------------------------------------------------------------------------------ Muon prologue
// Per stack of K matrices of `per` elements: g' = g * coef; mb = lerp(mb, g', 1-mom);
// x = bf16(lerp(g', mb, mom)); fro[k] += sum x^2.  (torch lerp formula.)
__device__ __forceinline__ float lerp_t(float a, float b, float w) {
  return (fabsf(w) < 0.5f) ? a + w * (b - a) : b - (b - a) * (1.f - w);
}

__global__ void muon_pre_kernel(const float* __restrict__ g, float* __restrict__ mb, __nv_bfloat16* __restrict__ x,
                                long long per, int K, const float* __restrict__ coef_ptr,
                                const float* __restrict__ mom_ptr, const float* __restrict__ one_mom_ptr,
                                float* __restrict__ fro) {
  const int k = blockIdx.y;
  const float coef = coef_ptr ? *coef_ptr : 1.f;
  const float mom = *mom_ptr, one_mom = *one_mom_ptr;
  const long long base = (long long)k * per;
  float ss = 0.f;
  for (long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < per;
       i += (long long)gridDim.x * blockDim.x * 4) {
    const float4 gv = *reinterpret_cast<const float4*>(g + base + i);
    float4 m = *reinterpret_cast<const float4*>(mb + base + i);
    const float ga[4] = {gv.x * coef, gv.y * coef, gv.z * coef, gv.w * coef};
    float ma[4] = {m.x, m.y, m.z, m.w};
    float xa[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ma[j] = lerp_t(ma[j], ga[j], one_mom);
      xa[j] = __bfloat162float(__float2bfloat16_rn(lerp_t(ga[j], ma[j], mom)));
      ss += xa[j] * xa[j];
    }
    *reinterpret_cast<float4*>(mb + base + i) = make_float4(ma[0], ma[1], ma[2], ma[3]);
    uint2 u;
    u.x = pack_bf16x2(xa[0], xa[1]);
    u.y = pack_bf16x2(xa[2], xa[3]);
    *reinterpret_cast<uint2*>(x + base + i) = u;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    // one partial per block, summed in block order by the consumer: the norm (and so the
    // whole Muon step) is bit-reproducible, which replicas that each run the optimizer on
    // identical gradients rely on
    fro[(long long)k * gridDim.x + blockIdx.x] = t;
  }
}

// ------------------------------------------------------------------------------ gather + apply
struct ApplyRun {
  int owner;            // rank whose update buffer holds this run
  long long src_off;    // element offset of the run in that buffer
  float* w;             // fp32 master (local)
  __nv_bfloat16* w16;   // bf16 cache (local), may be null
  long long n;          // elements
  const float* lr;      // device scalars
  const float* lrwd;
  long long blk0;       // first block index of this run
};

constexpr int kApplyChunk = 4096;

__global__ void symm_ag_apply_kernel(PeerBf16 upd, const ApplyRun* __restrict__ runs, int nruns) {
  const long long blk = blockIdx.x;
  int lo = 0, hi = nruns - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (runs[mid].blk0 <= blk) lo = mid;
    else hi = mid - 1;
  }
  const ApplyRun r = runs[lo];
  const long long start = (blk - r.blk0) * kApplyChunk;
  const long long end = min(start + (long long)kApplyChunk, r.n);
  const __nv_bfloat16* src = upd.p[r.owner] + r.src_off;
  const float lr_b = __bfloat162float(__float2bfloat16_rn(*r.lr));
  const float lrwd = *r.lrwd;
  // Two 8-element groups per thread, all loads issued before any math (memory-level
  // parallelism for the peer loads, which see NVLink latency).
  constexpr int kPer = kApplyChunk / 2;
  uint4 gu[2];
  float4 wl[2][2];
  bool ok[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const long long i = start + u * kPer + threadIdx.x * 8;
    ok[u] = i < end;
    if (ok[u]) {
      gu[u] = *reinterpret_cast<const uint4*>(src + i);
      wl[u][0] = *reinterpret_cast<const float4*>(r.w + i);
      wl[u][1] = *reinterpret_cast<const float4*>(r.w + i + 4);
    }
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (!ok[u]) continue;
    const long long i = start + u * kPer + threadIdx.x * 8;
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gu[u]);
    float wv[8] = {wl[u][0].x, wl[u][0].y, wl[u][0].z, wl[u][0].w, wl[u][1].x, wl[u][1].y, wl[u][1].z, wl[u][1].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 gf = __bfloat1622float2(g2[j]);
      const float gg[2] = {gf.x, gf.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float wi = wv[2 * j + e];
        const float t = __bfloat162float(__float2bfloat16_rn(lr_b * gg[e]));
        const float mask = (gg[e] * wi >= 0.f) ? 1.f : 0.f;
        wv[2 * j + e] = wi - (t + lrwd * wi * mask);
      }
    }
    *reinterpret_cast<float4*>(r.w + i) = make_float4(wv[0], wv[1], wv[2], wv[3]);
    *reinterpret_cast<float4*>(r.w + i + 4) = make_float4(wv[4], wv[5], wv[6], wv[7]);
    if (r.w16) {
      uint4 q;
      q.x = pack_bf16x2(wv[0], wv[1]);
      q.y = pack_bf16x2(wv[2], wv[3]);
      q.z = pack_bf16x2(wv[4], wv[5]);
      q.w = pack_bf16x2(wv[6], wv[7]);
      *reinterpret_cast<uint4*>(r.w16 + i) = q;
    }
  }
}

// ------------------------------------------------------------------------------ host
template <typename P, typename T>
static P peers_of(const std::vector<int64_t>& ptrs) {
  TORCH_CHECK((int)ptrs.size() <= kMaxRanks && !ptrs.empty(), "1..8 ranks");
  P p{};
  for (size_t i = 0; i < ptrs.size(); ++i) p.p[i] = reinterpret_cast<T>(ptrs[i]);
  return p;
}

void symm_barrier(std::vector<int64_t> pad_ptrs, int64_t rank, int64_t epoch, torch::Tensor err) {
  auto pads = peers_of<PeerU32, uint32_t*>(pad_ptrs);
  symm_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(pads, (int)rank, (int)pad_ptrs.size(),
                                                                       (uint32_t)epoch, err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// peer_ptrs: base addresses (fp32 elements) of every rank's gradient buffer
void symm_rs(std::vector<int64_t> peer_ptrs, int64_t src_off, int64_t n, torch::Tensor out, double inv,
             c10::optional<torch::Tensor> sumsq, int64_t mc_ptr) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= n, "out");
  TORCH_CHECK(n % 4 == 0 && src_off % 4 == 0, "16-byte granularity");
  auto peers = peers_of<PeerF32, const float*>(peer_ptrs);
  for (auto p : peer_ptrs) TORCH_CHECK((p & 15) == 0, "peer buffers must be 16-byte aligned");
  const float* mc = mc_ptr ? reinterpret_cast<const float*>(mc_ptr) : nullptr;
  const long long n4 = n / 4;
  const int blocks = (int)std::max<long long>(1, std::min<long long>((n4 + 255) / 256, 148 * 4));
  symm_rs_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      peers, (int)peer_ptrs.size(), src_off, n, out.data_ptr<float>(), (float)inv,
      sumsq.has_value() ? sumsq->data_ptr<float>() : nullptr, mc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// fro: fp32 [K, kMuonPreBlocks] partial sums of squares (every entry written).
void muon_pre(torch::Tensor g, torch::Tensor mb, torch::Tensor x, c10::optional<torch::Tensor> coef, torch::Tensor mom,
              torch::Tensor one_mom, torch::Tensor fro) {
  TORCH_CHECK(g.dim() == 3 && g.is_contiguous() && mb.is_contiguous() && x.is_contiguous(), "[K, r, c] stacks");
  const int K = (int)g.size(0);
  const long long per = g.size(1) * g.size(2);
  TORCH_CHECK(per % 4 == 0, "matrix size % 4");
  TORCH_CHECK(fro.scalar_type() == at::kFloat && fro.is_contiguous() && fro.numel() == (int64_t)K * kMuonPreBlocks,
              "fro fp32 [K, 64] partial sums");
  dim3 grid((unsigned)kMuonPreBlocks, K);
  muon_pre_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      g.data_ptr<float>(), mb.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), per, K,
      coef.has_value() ? coef->data_ptr<float>() : nullptr, mom.data_ptr<float>(), one_mom.data_ptr<float>(),
      fro.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// runs: int64 [nruns, 8] = owner, src_off, w_ptr, w16_ptr, n, lr_ptr, lrwd_ptr, unused.
// Runs are cut into pieces of kApplyPiece elements and the pieces are dealt round-robin
// over owners, so at every point of the grid the blocks in flight read a balanced mix of
// local and peer updates (the local half is HBM-bound, the peer half NVLink-bound; run
// back to back the two phases would not overlap).
constexpr long long kApplyPiece = 64LL * kApplyChunk;

void symm_ag_apply(std::vector<int64_t> upd_ptrs, torch::Tensor runs_i64) {
  TORCH_CHECK(runs_i64.scalar_type() == at::kLong && runs_i64.dim() == 2 && runs_i64.size(1) == 8 &&
                  runs_i64.device().is_cpu(),
              "runs table int64 [n, 8] on the host");
  auto upd = peers_of<PeerBf16, const __nv_bfloat16*>(upd_ptrs);
  const int nr = (int)runs_i64.size(0);
  const int64_t* t = runs_i64.data_ptr<int64_t>();
  std::vector<std::vector<ApplyRun>> by_owner(kMaxRanks);
  for (int i = 0; i < nr; ++i) {
    const int64_t* r = t + i * 8;
    TORCH_CHECK(r[4] % 8 == 0 && r[1] % 8 == 0, "runs must be multiples of 8 elements");
    TORCH_CHECK(r[0] >= 0 && r[0] < (int64_t)upd_ptrs.size(), "owner rank out of range");
    for (long long o = 0; o < r[4]; o += kApplyPiece) {
      const long long len = std::min<long long>(kApplyPiece, r[4] - o);
      by_owner[r[0]].push_back(ApplyRun{(int)r[0], r[1] + o, reinterpret_cast<float*>(r[2]) + o,
                                        r[3] ? reinterpret_cast<__nv_bfloat16*>(r[3]) + o : nullptr, len,
                                        reinterpret_cast<const float*>(r[5]), reinterpret_cast<const float*>(r[6]), 0});
    }
  }
  std::vector<ApplyRun> host;
  long long blocks = 0;
  for (size_t k = 0;; ++k) {
    bool any = false;
    for (auto& v : by_owner) {
      if (k < v.size()) {
        any = true;
        ApplyRun a = v[k];
        a.blk0 = blocks;
        blocks += (a.n + kApplyChunk - 1) / kApplyChunk;
        host.push_back(a);
      }
    }
    if (!any) break;
  }
  if (host.empty()) return;
  const size_t bytes = host.size() * sizeof(ApplyRun);
  auto tab = torch::empty({(long long)bytes}, torch::dtype(torch::kUInt8).pinned_memory(true));
  memcpy(tab.data_ptr(), host.data(), bytes);
  auto s = at::cuda::getCurrentCUDAStream();
  auto dtab = tab.to(torch::Device(torch::kCUDA, c10::cuda::current_device()), /*non_blocking=*/true);
  symm_ag_apply_kernel<<<(unsigned)blocks, 256, 0, s>>>(upd, reinterpret_cast<const ApplyRun*>(dtab.data_ptr()),
                                                        (int)host.size());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace tfb
