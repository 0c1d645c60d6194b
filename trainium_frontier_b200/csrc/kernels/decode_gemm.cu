// Decode-step linears: Y[M, N] = X[M, K] W[N, K]^T for the few rows of a KV-cache decode
// step (one token per sequence, M <= 128), with the step's elementwise work fused in.
//
// At these shapes the weights are the only large operand, so the kernel is laid out to
// stream them at HBM rate and to do nothing else on the critical path:
//  * swapped operands: the tcgen05 MMA's 128-row A side is a 128-row slab of W and its N
//    side the M activation rows (padded to 32 / 64 / 128), so no tensor-core work or
//    shared memory is spent on 128-row padding of X; the accumulator is 128 TMEM lanes
//    (weight rows) x Mpad fp32 columns (activation rows);
//  * split-K over a thread-block cluster of S CTAs (S in 1, 2, 4, 8): every CTA of a
//    cluster owns the same 128 weight rows and a slice of K; each CTA pushes the rows of
//    its partial tile that rank r finishes into rank r's shared memory with one bulk copy
//    (cp.async.bulk shared::cta -> shared::cluster, counted on rank r's mbarrier), and
//    rank r adds the S partials in rank order.  No fp32 workspace in global memory, no
//    atomics, nothing to re-zero between launches, so a captured CUDA graph replays it
//    as is;
//  * programmatic dependent launch: the weight slabs do not depend on the previous kernel,
//    so the producer issues their TMA loads before griddepcontrol.wait, and each CTA
//    triggers its dependents once its MMAs are done, so the next kernel's weight stream
//    overlaps this one's reduction and stores;
//  * fused epilogues on the reduced tile:
//      DEC_PLAIN  y
//      DEC_RES    y + R
//      DEC_RELU2  relu(bf16(y) - tau)^2
//      DEC_MIX    lambda_r * bf16(y + R) + lambda_0 * x0   (the next block's residual mix)
//      DEC_QKV    q / k heads: RoPE at the device-side position, then QK RMS norm; q rows
//                 to `out`, k and v rows straight into the KV cache at that position
//                 (token-major [B, T_max, H*128] or head-major [B, H, T_max, 128])
//    and, for any of them, a per-row RMS norm of the input (`row_norm`): by linearity
//    rsqrt(mean(x^2) + eps) scales the rows of X W^T, and every CTA adds the sums of
//    squares of its K slice of X to the cluster reduction.
//
// Warp roles (192 threads): warp 0 lane 0 TMA producer, warp 1 TMEM owner + MMA issuer,
// warps 2-5 epilogue (sums of squares, TMEM -> shared partial tile, the pushes, then the
// rows this CTA owns: rank r of the cluster finishes rows [r * mr, (r + 1) * mr), mr =
// ceil(M / S) rounded up to 4).  One cluster barrier, split into an arrive after set-up
// and a wait before the first push, guarantees every peer's mbarrier is initialised.
// Every wait is bounded (sm100_common.cuh).
//
// The ops fused here are the reference's per-block decode math (train.py:2564-2567
// attention inputs, train.py:2415-2420 rotary, train.py:1432-1433 norm, train.py:2218-2234
// relu^2 MLP, train.py:2652-2654 residual mix); the reference itself has no decode path.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

CUtensorMap make_tmap_bf16(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                           uint32_t box_inner, uint32_t box_outer, uint64_t batch, uint64_t batch_stride_elems);
int num_sms(int dev);
void cache_strides(const torch::Tensor& c, int64_t H, int64_t D, long long& sb, long long& sh, long long& st,
                   int& tmax);

enum : int { DEC_PLAIN = 0, DEC_RES = 1, DEC_RELU2 = 2, DEC_MIX = 3, DEC_QKV = 4 };

constexpr int kDgBM = 128;                  // weight rows per tile (the MMA's M)
constexpr int kDgBK = 64;                   // K per stage: one 128-byte swizzled row
constexpr int kDgWBytes = kDgBM * kDgBK * 2;  // 16 KB of weights per stage
constexpr int kDgThreads = 192;
constexpr int kDgMaxSplit = 8;
constexpr float kDgNormEps = 1.1920928955078125e-07f;  // F.rms_norm's default for fp32 math

struct DecGemmArgs {
  int M, N, K, Mpad;
  int kb_total, S, mr;
  int epi, row_norm;
  const __nv_bfloat16* X;  // the TMA operand, also read directly for the sums of squares
  long long ldx;
  const __nv_bfloat16* R;
  long long ldr;
  const __nv_bfloat16* X0;
  long long ldx0;
  const float* lam_r;
  const float* lam_0;
  float tau;
  __nv_bfloat16* out;
  long long ldo;
  // DEC_QKV: W rows are [q heads | k heads | v heads] x 128, out receives the q rows
  int H;
  const __nv_bfloat16* cosb;  // [positions, 64]
  const __nv_bfloat16* sinb;
  const int* pos_ptr;
  __nv_bfloat16* kc;  // [B, Tmax, H * 128] or [B, H, Tmax, 128]: strides (batch, head, token)
  __nv_bfloat16* vc;
  long long cs_b, cs_h, cs_t;
  int Tmax;
  int* err;
  unsigned long long* trace;  // optional phase timeline (globaltimer ns) of the first and last CTA
};

// Phase timeline (off unless a buffer is installed with decode_gemm_trace_set): the first
// and the last CTA of the grid write %globaltimer at each phase into trace[slot * 16 + e].
//   0 entry, 1 set-up done, 2 weight loads issued, 3 grid dependency resolved (producer),
//   4 first stage landed (MMA), 5 last MMA issued, 6 sums of squares done, 7 MMAs complete
//   (epilogue), 8 partial tile in shared memory, 9 pushes to the owners issued,
//   10 every peer's partials received, 11 rows finished and pushes read
__device__ __forceinline__ void dg_stamp(unsigned long long* tr, int e) {
  if (tr == nullptr) return;
  const unsigned last = gridDim.x - 1;
  if (blockIdx.x == 0 || blockIdx.x == last) tr[(blockIdx.x == 0 ? 0 : 16) + e] = globaltimer_ns();
}

__device__ __forceinline__ float dg_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory to another CTA's
// (dst and mbar: shared::cluster addresses); completion counted on that CTA's mbarrier.
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(mbar)
               : "memory");
}

template <int STAGES>
__global__ void __launch_bounds__(kDgThreads, 1)
    decode_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                       const __grid_constant__ DecGemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int XB = a.Mpad * 128;  // bytes of one X stage (Mpad rows x 64 bf16)
  const int S = a.S, mr = a.mr;  // cluster size; rows finished per rank (a multiple of 4)
  uint8_t* sW = smem;
  uint8_t* sX = smem + STAGES * kDgWBytes;
  // [S * mr][128] fp32 partial tile of this CTA's K slice; reuses the weight ring once
  // every MMA of this CTA has read it
  float* part = reinterpret_cast<float*>(smem);
  float* recv = reinterpret_cast<float*>(sX + STAGES * XB);  // [S][mr][128] partials of this rank's rows
  float* rssq = recv + S * mr * kDgBM;                       // [S][mr] their sums of squares
  float* ssq = rssq + S * mr;                                // [132] this K slice's sums of squares
  float* scratch = ssq + 132;                                // [16] QK-norm cross-warp sums
  uint64_t* full = reinterpret_cast<uint64_t*>(scratch + 16);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint64_t* drain = done + 1;
  uint64_t* recv_bar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int crank = (int)cluster_ctarank();
  const int nb = (int)cluster_id_x();
  const int kb0 = (int)((long long)crank * a.kb_total / S);
  const int kb1 = (int)((long long)(crank + 1) * a.kb_total / S);
  const int nk = kb1 - kb0;
  const uint32_t tcols = (uint32_t)a.Mpad;  // 32, 64 or 128: a power of two >= 32
  const int m_lo = crank * mr, m_hi = min(a.M, m_lo + mr);  // rows this rank finishes
  const bool owner = m_lo < a.M;
  // every sender pushes mr rows of partials (+ mr sums of squares) to each owner
  const uint32_t push_bytes = (uint32_t)(mr * kDgBM * 4 + (a.row_norm ? mr * 4 : 0));
  if (threadIdx.x == 0) dg_stamp(a.trace, 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(drain, 1);
    mbar_init(recv_bar, 1);
    // the phase completes once this arrival and every peer's pushed bytes are in
    if (owner) mbar_arrive_expect_tx(recv_bar, (uint32_t)S * push_bytes);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tcols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // this CTA's barriers are initialised: peers may push into it once they have waited
  cluster_arrive_release();
  if (threadIdx.x == 0) dg_stamp(a.trace, 1);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const int pre = nk < STAGES ? nk : STAGES;
      uint32_t out_valid = 0, out_parity = 0;
      bool ok = true;
      // weights first: they do not depend on the previous kernel of the stream
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], (uint32_t)(kDgWBytes + XB));
        out_valid |= 1u << i;
        tma_load_3d(sW + i * kDgWBytes, &tmW, &full[i], (kb0 + i) * kDgBK, nb * kDgBM, 0);
      }
      dg_stamp(a.trace, 2);
      griddep_wait();
      dg_stamp(a.trace, 3);
      for (int i = 0; i < pre; ++i) tma_load_3d(sX + i * XB, &tmX, &full[i], (kb0 + i) * kDgBK, 0, 0);
      for (int i = pre; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)((i / STAGES) & 1);
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, a.err, ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], (uint32_t)(kDgWBytes + XB));
        out_parity = (out_parity & ~(1u << s)) | (ph << s);
        tma_load_3d(sW + s * kDgWBytes, &tmW, &full[s], (kb0 + i) * kDgBK, nb * kDgBM, 0);
        tma_load_3d(sX + s * XB, &tmX, &full[s], (kb0 + i) * kDgBK, 0, 0);
      }
      if (!ok) {
        *abort_flag = 1;
        // no bulk copy may still be writing shared memory when the CTA exits
        for (int s = 0; s < STAGES; ++s) {
          if (!((out_valid >> s) & 1u)) continue;
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], (out_parity >> s) & 1u)) {
            if (globaltimer_ns() - t0 > 100000000ull) break;
          }
        }
      }
    }
    __syncwarp();
    cluster_wait_acquire();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kDgBM, a.Mpad, false, false);
      bool ok = true;
      griddep_wait();  // the bounded waits below then time this kernel's loads, not its predecessor
      for (int i = 0; i < nk; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)((i / STAGES) & 1);
        if (!mbar_wait(&full[s], ph, abort_flag, a.err, ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        if (i == 0) dg_stamp(a.trace, 4);
        tc_fence_after();
        const uint32_t wa = smem_u32(sW + s * kDgWBytes), xa = smem_u32(sX + s * XB);
#pragma unroll
        for (int kk = 0; kk < kDgBK / 16; ++kk)
          umma_bf16(tmem_base, umma_desc_sw128(wa + kk * 32, 16, 1024), umma_desc_sw128(xa + kk * 32, 16, 1024),
                    idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      // arrives once every MMA issued above has completed (at once if there were none)
      umma_commit(done);
      dg_stamp(a.trace, 5);
      if (!ok) *abort_flag = 1;
    }
    __syncwarp();
    cluster_wait_acquire();
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int et = threadIdx.x - 64;
    griddep_wait();
    if (a.row_norm) {
      // warp ew sums rows ew, ew + 4, ...; eight rows' loads are issued together so the
      // pass costs one memory round trip per 256 columns, not one per row
      const int c0 = kb0 * kDgBK, c1 = min(kb1 * kDgBK, a.K);
      for (int m0 = ew; m0 < a.Mpad; m0 += 4 * 8) {
        float s[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) s[r] = 0.f;
        for (int c = c0 + lane * 8; c < c1; c += 256) {
          uint4 u[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const int m = m0 + 4 * r;
            u[r] = m < a.M ? *reinterpret_cast<const uint4*>(a.X + (long long)m * a.ldx + c) : make_uint4(0u, 0u, 0u, 0u);
          }
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u[r]);
#pragma unroll
            for (int q2 = 0; q2 < 4; ++q2) {
              const float2 f = __bfloat1622float2(h2[q2]);
              s[r] += f.x * f.x + f.y * f.y;
            }
          }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float t = dg_warp_sum(s[r]);
          if (lane == 0 && m0 + 4 * r < a.Mpad) ssq[m0 + 4 * r] = t;
        }
      }
    }
    if (threadIdx.x == 64) dg_stamp(a.trace, 6);
    const bool ok = mbar_wait_warp(done, 0, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE);
    if (threadIdx.x == 64) dg_stamp(a.trace, 7);
    tc_fence_after();
    {
      const int q = warp & 3;  // the TMEM lane quarter this warp may read
      const int n = q * 32 + lane;
      for (int c0 = 0; c0 < a.Mpad; c0 += 32) {
        uint32_t r[32];
        if (ok && nk > 0) {
          tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) r[jj] = 0u;
        }
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) part[(c0 + jj) * kDgBM + n] = __uint_as_float(r[jj]);
      }
    }
    tc_fence_before();
    fence_proxy_async_smem();  // the bulk copies below read `part` / `ssq` through the async proxy
    named_bar_sync(1, 128);
    griddep_launch_dependents();
    if (threadIdx.x == 64) dg_stamp(a.trace, 8);
    cluster_wait_acquire();  // every peer's barriers are initialised
    if (threadIdx.x == 64) {
      // push rows [r * mr, r * mr + mr) of the partial tile (and their sums of squares) to
      // rank r, into its slot for this rank; completion counts on rank r's recv_bar
      for (int r = 0; r < S; ++r) {
        if (r * mr >= a.M) break;
        const uint32_t rbar = mapa_shared(smem_u32(recv_bar), (uint32_t)r);
        bulk_copy_to_peer(mapa_shared(smem_u32(recv + (size_t)crank * mr * kDgBM), (uint32_t)r),
                          part + (size_t)r * mr * kDgBM, (uint32_t)(mr * kDgBM * 4), rbar);
        if (a.row_norm)
          bulk_copy_to_peer(mapa_shared(smem_u32(rssq + crank * mr), (uint32_t)r), ssq + r * mr, (uint32_t)(mr * 4), rbar);
      }
      bulk_commit_group();
      dg_stamp(a.trace, 9);
    }

    // ---------------------------------------------------------- finish this rank's rows
    const int slot = et >> 6, j = et & 63;  // two rows at a time, thread pair (j, j + 64)
    const int n0 = nb * kDgBM;
    const int ca = n0 + j, cb = n0 + j + 64;
    const bool va = ca < a.N, vb = cb < a.N;
    int pos = 0;
    if (a.epi == DEC_QKV) pos = *a.pos_ptr;
    float lr = 1.f, l0 = 0.f;
    if (a.epi == DEC_MIX) {
      lr = *a.lam_r;
      l0 = *a.lam_0;
    }
    constexpr int U = 4;
    float ra[U], rb[U], xa[U], xb[U];
    // residual / x0 values of a batch of U rows (issued before the partials are awaited)
    auto load_rows = [&](int mb) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int m = mb + 2 * u;
        ra[u] = rb[u] = xa[u] = xb[u] = 0.f;
        if (m < m_hi && (a.epi == DEC_RES || a.epi == DEC_MIX)) {
          const __nv_bfloat16* rrow = a.R + (long long)m * a.ldr;
          if (va) ra[u] = __bfloat162float(rrow[ca]);
          if (vb) rb[u] = __bfloat162float(rrow[cb]);
        }
        if (m < m_hi && a.epi == DEC_MIX) {
          const __nv_bfloat16* x0row = a.X0 + (long long)m * a.ldx0;
          if (va) xa[u] = __bfloat162float(x0row[ca]);
          if (vb) xb[u] = __bfloat162float(x0row[cb]);
        }
      }
    };
    if (owner) {
      load_rows(m_lo + slot);
      mbar_wait_warp(recv_bar, 0, abort_flag, a.err, ERR_TIMEOUT_PEER);
      // one decision for all four warps (the QKV path has named barriers per warp pair)
      named_bar_sync(1, 128);
      const bool got = *abort_flag == 0;
      if (threadIdx.x == 64) dg_stamp(a.trace, 10);
      for (int mb = m_lo + slot; mb < m_hi && got; mb += 2 * U) {
        if (mb != m_lo + slot) load_rows(mb);
        float v0[U], v1[U], ss[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          v0[u] = v1[u] = ss[u] = 0.f;
          const int ml = mb + 2 * u - m_lo;
          if (ml + m_lo < m_hi) {
#pragma unroll
            for (int p = 0; p < kDgMaxSplit; ++p) {
              if (p < S) {  // rank order: the sum is the same on every launch
                const float* src = recv + ((size_t)p * mr + ml) * kDgBM;
                v0[u] += src[j];
                v1[u] += src[j + 64];
                if (a.row_norm) ss[u] += rssq[p * mr + ml];
              }
            }
          }
        }
        if (a.row_norm) {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const float rs = rsqrtf(ss[u] / (float)a.K + kDgNormEps);
            v0[u] *= rs;
            v1[u] *= rs;
          }
        }
        if (a.epi != DEC_QKV) {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int m = mb + 2 * u;
            if (m >= m_hi) continue;
            float y0 = v0[u], y1 = v1[u];
            if (a.epi == DEC_RES) {
              y0 += ra[u];
              y1 += rb[u];
            } else if (a.epi == DEC_RELU2) {
              const float h0 = bf16r(y0) - a.tau, h1 = bf16r(y1) - a.tau;
              y0 = h0 > 0.f ? h0 * h0 : 0.f;
              y1 = h1 > 0.f ? h1 * h1 : 0.f;
            } else if (a.epi == DEC_MIX) {
              y0 = lr * bf16r(y0 + ra[u]) + l0 * xa[u];
              y1 = lr * bf16r(y1 + rb[u]) + l0 * xb[u];
            }
            __nv_bfloat16* orow = a.out + (long long)m * a.ldo;
            if (va) orow[ca] = __float2bfloat16_rn(y0);
            if (vb) orow[cb] = __float2bfloat16_rn(y1);
          }
        } else {  // DEC_QKV (128-wide heads, one head per tile)
          const bool in_cache = pos >= 0 && pos < a.Tmax;
          if (nb < 2 * a.H) {
            const int tp = in_cache ? pos : 0;  // table row (out-of-range positions write no cache row)
            const float c = __bfloat162float(a.cosb[(long long)tp * 64 + j]);
            const float sn = __bfloat162float(a.sinb[(long long)tp * 64 + j]);
            float y1[U], y2[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const float x1 = bf16r(v0[u]), x2 = bf16r(v1[u]);
              y1[u] = x1 * c + x2 * sn;
              y2[u] = x2 * c - x1 * sn;
              const float t = dg_warp_sum(y1[u] * y1[u] + y2[u] * y2[u]);
              if (lane == 0) scratch[(slot * 2 + (warp & 1)) * U + u] = t;
            }
            named_bar_sync(2 + slot, 64);
            float tot[U];
#pragma unroll
            for (int u = 0; u < U; ++u) tot[u] = scratch[(slot * 2) * U + u] + scratch[(slot * 2 + 1) * U + u];
            named_bar_sync(2 + slot, 64);
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const int m = mb + 2 * u;
              if (m >= m_hi) continue;
              const float r = rsqrtf(tot[u] / 128.f + kDgNormEps);
              const __nv_bfloat16 z1 = __float2bfloat16_rn(y1[u] * r), z2 = __float2bfloat16_rn(y2[u] * r);
              if (nb < a.H) {
                __nv_bfloat16* orow = a.out + (long long)m * a.ldo;
                orow[nb * 128 + j] = z1;
                orow[nb * 128 + j + 64] = z2;
              } else if (in_cache) {
                __nv_bfloat16* kr = a.kc + (long long)m * a.cs_b + (long long)pos * a.cs_t + (long long)(nb - a.H) * a.cs_h;
                kr[j] = z1;
                kr[j + 64] = z2;
              }
            }
          } else if (in_cache) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const int m = mb + 2 * u;
              if (m >= m_hi) continue;
              __nv_bfloat16* vr = a.vc + (long long)m * a.cs_b + (long long)pos * a.cs_t + (long long)(nb - 2 * a.H) * a.cs_h;
              vr[j] = __float2bfloat16_rn(bf16r(v0[u]));
              vr[j + 64] = __float2bfloat16_rn(bf16r(v1[u]));
            }
          }
        }
      }
    }
    if (threadIdx.x == 64) {
      bulk_wait_group_read<0>();  // the pushes have read `part` before the CTA's memory is released
      dg_stamp(a.trace, 11);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tcols);
  }
}

// ------------------------------------------------------------------------ host side
static unsigned long long* g_dg_trace = nullptr;

// Install (or with None remove) a uint64 [32] buffer that the next decode GEMM launches
// fill with the phase timeline of their first and last CTA (see dg_stamp).
void decode_gemm_trace_set(c10::optional<torch::Tensor> buf) {
  if (buf.has_value()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->numel() >= 32, "int64 [32]");
    g_dg_trace = reinterpret_cast<unsigned long long*>(buf->data_ptr<int64_t>());
  } else {
    g_dg_trace = nullptr;
  }
}

static size_t dg_smem_bytes(int stages, int mpad, int S, int mr) {
  return 1024 + (size_t)stages * (kDgWBytes + (size_t)mpad * 128) + (size_t)S * mr * (kDgBM * 4 + 4) + 132 * 4 + 16 * 4 +
         (2 * stages + 3) * 8 + 16;
}

template <int STAGES>
static void dg_launch(const CUtensorMap& tw, const CUtensorMap& tx, const DecGemmArgs& a, int tiles, bool pdl,
                      cudaStream_t stream) {
  auto kern = decode_gemm_kernel<STAGES>;
  const size_t smem = dg_smem_bytes(STAGES, a.Mpad, a.S, a.mr);
  TORCH_CHECK(smem <= 232448, "decode GEMM shared memory above the per-CTA limit");
  // the partial tile ([max(Mpad, S * mr)][128] fp32) reuses the weight + activation rings
  TORCH_CHECK((size_t)std::max(a.Mpad, a.S * a.mr) * kDgBM * 4 <= (size_t)STAGES * (kDgWBytes + (size_t)a.Mpad * 128),
              "decode GEMM: pipeline too shallow to hold the partial tile");
  static int smem_set = 0;
  if ((int)smem > smem_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    smem_set = (int)smem;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)(tiles * a.S), 1, 1);
  cfg.blockDim = dim3(kDgThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, tw, tx, a));
}

// out[M, N] (bf16) = epilogue(X[M, K] W[N, K]^T); see the file comment for `epi`.
// split = 0 picks the cluster size and pipeline depth from the shape; pdl = launch with
// programmatic stream serialization (the kernel waits on griddepcontrol before it reads
// anything an earlier kernel of the stream wrote).
void decode_gemm(torch::Tensor X, torch::Tensor W, torch::Tensor out, int64_t epi, bool row_norm,
                 c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> X0, c10::optional<torch::Tensor> lam_r,
                 c10::optional<torch::Tensor> lam_0, double tau, c10::optional<torch::Tensor> cos,
                 c10::optional<torch::Tensor> sin, c10::optional<torch::Tensor> pos, c10::optional<torch::Tensor> kc,
                 c10::optional<torch::Tensor> vc, int64_t H, int64_t split, bool pdl, torch::Tensor err) {
  TORCH_CHECK(X.is_cuda() && W.is_cuda() && out.is_cuda() && X.dim() == 2 && W.dim() == 2 && out.dim() == 2,
              "2-D CUDA operands");
  TORCH_CHECK(X.scalar_type() == at::kBFloat16 && W.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16,
              "bf16 operands");
  TORCH_CHECK(X.stride(1) == 1 && W.stride(1) == 1 && out.stride(1) == 1, "row-major operands");
  const int64_t M = X.size(0), K = X.size(1), N = W.size(0);
  TORCH_CHECK(M >= 1 && M <= 128, "decode GEMM serves 1..128 rows");
  TORCH_CHECK(W.size(1) == K && K % 8 == 0, "K mismatch or K not a multiple of 8");
  TORCH_CHECK((X.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(X.data_ptr()) & 15) == 0,
              "X rows must be 16-byte aligned");
  TORCH_CHECK(epi >= DEC_PLAIN && epi <= DEC_QKV, "unknown epilogue");
  DecGemmArgs a{};
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.Mpad = M <= 32 ? 32 : (M <= 64 ? 64 : 128);
  a.kb_total = (int)((K + kDgBK - 1) / kDgBK);
  a.epi = (int)epi;
  a.row_norm = row_norm ? 1 : 0;
  a.X = reinterpret_cast<const __nv_bfloat16*>(X.data_ptr());
  a.ldx = X.stride(0);
  a.tau = (float)tau;
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ldo = out.stride(0);
  a.err = err.data_ptr<int>();
  auto bf_rows = [&](const torch::Tensor& t, const char* what) {
    TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2 && t.stride(1) == 1 &&
                    t.size(0) >= M && t.size(1) >= N,
                what, " must be bf16 [M, N] rows");
  };
  if (epi == DEC_RES || epi == DEC_MIX) {
    TORCH_CHECK(R.has_value(), "residual required");
    bf_rows(*R, "R");
    a.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr());
    a.ldr = R->stride(0);
  }
  if (epi == DEC_MIX) {
    TORCH_CHECK(X0.has_value() && lam_r.has_value() && lam_0.has_value(), "mix needs x0 and both lambdas");
    bf_rows(*X0, "x0");
    TORCH_CHECK(lam_r->scalar_type() == at::kFloat && lam_0->scalar_type() == at::kFloat, "fp32 lambdas");
    a.X0 = reinterpret_cast<const __nv_bfloat16*>(X0->data_ptr());
    a.ldx0 = X0->stride(0);
    a.lam_r = lam_r->data_ptr<float>();
    a.lam_0 = lam_0->data_ptr<float>();
  }
  if (epi == DEC_QKV) {
    TORCH_CHECK(cos.has_value() && sin.has_value() && pos.has_value() && kc.has_value() && vc.has_value(),
                "QKV epilogue needs cos, sin, pos and both caches");
    TORCH_CHECK(H >= 1 && N == 3 * H * 128, "QKV epilogue: W is [3 * H * 128, K] (head_dim 128)");
    TORCH_CHECK(kc->sizes() == vc->sizes() && kc->strides() == vc->strides() && kc->size(0) >= M &&
                    kc->scalar_type() == at::kBFloat16 && vc->scalar_type() == at::kBFloat16,
                "bf16 caches of one shape");
    long long sb, sh, st;
    int tmax;
    cache_strides(*kc, H, 128, sb, sh, st, tmax);
    TORCH_CHECK(cos->is_contiguous() && sin->is_contiguous() && cos->size(-1) == 64 && sin->size(-1) == 64,
                "rotary tables [positions, 64]");
    TORCH_CHECK(out.size(0) >= M && out.size(1) >= H * 128, "out receives q [M, H * 128]");
    a.H = (int)H;
    a.cosb = reinterpret_cast<const __nv_bfloat16*>(cos->data_ptr());
    a.sinb = reinterpret_cast<const __nv_bfloat16*>(sin->data_ptr());
    a.pos_ptr = pos->data_ptr<int>();
    a.kc = reinterpret_cast<__nv_bfloat16*>(kc->data_ptr());
    a.vc = reinterpret_cast<__nv_bfloat16*>(vc->data_ptr());
    a.cs_b = sb;
    a.cs_h = sh;
    a.cs_t = st;
    a.Tmax = (int)std::min<int64_t>(tmax, cos->numel() / 64);
  } else {
    TORCH_CHECK(out.size(0) >= M && out.size(1) >= N, "out [M, N]");
  }
  c10::cuda::CUDAGuard guard(X.device());
  const int tiles = (int)((N + kDgBM - 1) / kDgBM);
  const int sms = num_sms(X.get_device());
  // Pipeline depth and cluster size: few weight tiles -> 10 stages, one CTA per SM and
  // 8-way split-K (long K); otherwise 4 stages (two CTAs per SM when Mpad is 32) and the
  // widest split that fits one wave.
  // Pipeline depth: 3 stages, two CTAs per SM, and the widest split-K that fits one wave.
  // Measured on the d20 decode step (batch 32, 50 graph replays): 3 stages 1.113 ms,
  // 2: 1.121, 4: 1.212, 6: 1.104 (one CTA per SM); a "deep" mode (10 stages, one CTA per
  // SM, 8-way split for few-tile shapes) 1.325, because a CTA that fills an SM leaves no
  // room for the next kernel's CTAs to launch early under programmatic dependent launch.
  // TFB_DG_STAGES / TFB_DG_DEEP_STAGES (0 = off) override (2, 3, 4, 6, 8 or 10).
  static const int env_stages = [] {
    const char* e = getenv("TFB_DG_STAGES");
    return e ? atoi(e) : 3;
  }();
  static const int env_deep = [] {
    const char* e = getenv("TFB_DG_DEEP_STAGES");
    return e ? atoi(e) : 0;
  }();
  const bool deep = env_deep > 0 && (int64_t)tiles * kDgMaxSplit <= sms && a.Mpad <= 32;
  const int stages = deep ? env_deep : env_stages;
  const size_t smem_est = dg_smem_bytes(stages, a.Mpad, kDgMaxSplit, 16);
  const int slots = sms * std::max<int>(1, (int)std::min<size_t>(2, 228 * 1024 / (smem_est + 1024)));
  int S = 1;
  if (split > 0) {
    TORCH_CHECK(split == 1 || split == 2 || split == 4 || split == 8, "split must be 1, 2, 4 or 8");
    S = (int)split;
  } else {
    while (S < kDgMaxSplit && (int64_t)tiles * S * 2 <= slots && S * 2 <= a.kb_total) S *= 2;
  }
  a.trace = g_dg_trace;
  TORCH_CHECK(S <= a.kb_total, "more K splits than K blocks");
  a.S = S;
  a.mr = (int)(((M + S - 1) / S + 3) / 4 * 4);  // rows per rank, a multiple of 4 (16-byte pushes)
  TORCH_CHECK((int64_t)S * a.mr <= 128, "row split");
  const CUtensorMap tw = make_tmap_bf16(W.data_ptr(), K, N, W.stride(0), kDgBK, kDgBM, 1, 0);
  const CUtensorMap tx = make_tmap_bf16(X.data_ptr(), K, M, X.stride(0), kDgBK, (uint32_t)a.Mpad, 1, 0);
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (stages) {
    case 2: dg_launch<2>(tw, tx, a, tiles, pdl, stream); break;
    case 3: dg_launch<3>(tw, tx, a, tiles, pdl, stream); break;
    case 4: dg_launch<4>(tw, tx, a, tiles, pdl, stream); break;
    case 6: dg_launch<6>(tw, tx, a, tiles, pdl, stream); break;
    case 8: dg_launch<8>(tw, tx, a, tiles, pdl, stream); break;
    case 10: dg_launch<10>(tw, tx, a, tiles, pdl, stream); break;
    default: TORCH_CHECK(false, "decode GEMM pipeline depth must be 2, 3, 4, 6, 8 or 10");
  }
}

}  // namespace tfb
