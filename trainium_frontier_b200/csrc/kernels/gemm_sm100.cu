// Persistent warp-specialized bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   D[m, n] = epilogue( sum_k A[m, k] * B[n, k] )
//
// Operands are staged global -> shared memory by TMA (128-byte swizzle, K-major or
// MN-major for either operand, so all three products of a linear layer -- y = x W^T,
// dx = dy W and dW = dy^T x -- read their operands in place, with no transposes),
// multiplied by tcgen05.mma issued from one thread, accumulated in TMEM (fp32,
// double-buffered: the epilogue drains tile i while the MMAs of tile i+1 run) and
// read back with tcgen05.ld for a fused epilogue.
//
// CTA = 10 warps (12 with the all-gather copy warps), one CTA per SM, grid = min(#tiles, #SMs):
//   warp 0      TMA producer            (full[s] <- TMA bytes, waits empty[s])
//   warp 1      TMEM owner + MMA issuer (waits full[s], commits empty[s] / tfull[a])
//   warps 2..9  epilogue: warp w drains TMEM lane quarter (w & 3), column half (w - 2) >> 2
//               (waits tfull[a], arrives tempty[a]); two warps per quarter halve the
//               drain time, which short-K tiles would otherwise wait on
// Tile 128 x BN x 64 (BN = 256 or 128), 4 or 6 pipeline stages.
//
// Epilogues (the fused ops the model needs):
//   EPI_BF16      D = bf16(alpha * acc (+ R))               linear, linear + residual
//   EPI_ROPE      D = bf16(acc), then RoPE + per-head RMSNorm of the leading columns
//                 (fused QKV projection: q / k heads normalised, v stored as is)
//   EPI_RELU2     D2 = bf16(acc) (pre-activation h), D = bf16(relu(h - tau)^2)
//   EPI_RELU2_BWD D = bf16(bf16(alpha * acc) * 2 relu(R - tau))   (R = h)
//   EPI_F32       D(f32) = alpha * acc (+ D if beta)        weight gradients (fp32, split-K via
//                                                          vector atomics into the gradient)
//   EPI_CE        lm_head + logit softcap + cross-entropy statistics: z = bf16(acc) (stored
//                 only when the gradient is wanted), y = S tanh(z / S); each tile writes its
//                 rows' partial sums of exp(y - S) (one per tile column half) and the
//                 target's y to small per-row buffers, so no pass over the [tokens, vocab]
//                 logits is needed for the loss; ce_finish_kernel then adds the partials,
//                 writes the losses and (with the gradient) turns z into dz in one pass.
// Modes (the tensor-parallel collectives fused into the GEMM, over NVLink peer memory):
//   MODE_PLAIN    the GEMM above.
//   MODE_AG       all-gather -> GEMM.  A is the [M, K] gather buffer of which every rank
//                 of the tensor-parallel group owns rows_per_rank rows (its sequence
//                 shard, written there by the producing kernel).  Two extra copy warps
//                 pull the peers' rows over NVLink into this GPU's buffer, 128 rows at
//                 a time, while the MMAs start on the local rows; the TMA producer waits
//                 (bounded) on a per-m-block "copied" word before loading a remote
//                 m-block.  Every remote byte crosses NVLink once, and TMA only ever
//                 reads this GPU's own memory.
//   MODE_RS       GEMM -> reduce-scatter.  D = sum over ranks of the partial products,
//                 scattered by row owner.  Tiles of the peers' rows come first: their
//                 partials (bf16, staged through shared memory so they leave as whole
//                 128-byte row segments) are stored straight into the owner's receive
//                 buffer (P2P stores) and announced per tile and TMEM lane quarter with a
//                 release flag; tiles of this rank's rows come last and add the peers'
//                 partials (acquire-waited, bounded) and the residual in the epilogue.
// In the TP modes tiles are handed out dynamically (an atomic counter read by the
// producer, passed to the MMA and epilogue warps through a 4-slot ring in shared
// memory), so a tile that waits is only ever claimed after every tile that others wait
// for has been claimed by a running CTA: no wait depends on co-residency.
// Every TMA load is a plain per-CTA load of this GPU's own memory.
// Reference counterparts: Linear (train.py:2237-2267), relu^2 (train.py:1465-1515), the
// Newton-Schulz matmul chain (train.py:3629-3636).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

enum GemmEpi : int { EPI_BF16 = 0, EPI_RELU2 = 1, EPI_RELU2_BWD = 2, EPI_F32 = 3, EPI_ROPE = 4, EPI_CE = 5 };
enum GemmMode : int { MODE_PLAIN = 0, MODE_AG = 1, MODE_RS = 2 };

constexpr int kTpMaxRanks = 8;

struct TpArgs {
  int rank, world, rows_per_rank;  // rows of the full M range owned by each rank (multiple of 128)
  uint32_t epoch;                  // call index, identical on every rank of the group
  // all-gather side
  const uint8_t* ag_src[kTpMaxRanks];  // every rank's gather buffer
  uint8_t* ag_dst;                     // this rank's gather buffer
  long long ag_ld_bytes;               // row stride of the gather buffers (bytes)
  int ag_row_bytes;                    // bytes copied per row (K * 2)
  uint32_t* ag_ready[kTpMaxRanks];     // every rank's ready pad; word s is written by rank s
  uint32_t* ag_claim;                  // local claim word per remote m-block job
  uint32_t* ag_done;                   // local "copied" word per m-block
  // reduce-scatter side
  __nv_bfloat16* rs_recv[kTpMaxRanks];  // every rank's receive buffer [world][rows_per_rank][N] bf16
  uint32_t* rs_flag[kTpMaxRanks];      // every rank's flags [world][tiles per rank][8]
  uint32_t* sched;                     // local [2]: tile counter, finished-CTA counter
};

struct GemmArgs {
  int M, N, K;
  int tiles_m, tiles_n, split_k, kb_total, kb_per_split, num_tiles, batch;
  float alpha, beta, tau, rcoef;
  const float* alpha_ptr;  // optional device scalar multiplied into alpha
  void* D;
  long long ldd, d_bstride;
  void* D2;
  long long ldd2, d2_bstride;
  const __nv_bfloat16* R;
  long long ldr, r_bstride;
  int* err;
  int tma_store;  // bf16 outputs leave through TMA stores of staged 32 x 64 slabs
  // split-K finish (EPI_F32 with split_k > 1): the last split to add into a warp's region
  // of the fp32 workspace D writes bf16(D (+ rcoef R) | relu2(D)) to fin_out and re-zeroes D
  __nv_bfloat16* fin_out;
  long long ld_fin;
  int* fin_cnt;
  int fin_relu2;
  // EPI_ROPE: RoPE + per-head RMSNorm of the leading rope_cols columns (BN = 256, head_dim
  // 128: one epilogue warp's column half is one head, one thread one token of it)
  const __nv_bfloat16* rope_cos;  // [T][64] bf16, row = position
  const __nv_bfloat16* rope_sin;
  int rope_T, rope_cols, rope_heads;
  float* rope_rstd;  // [M][rope_heads] fp32, optional
  // EPI_CE (2-D, N = padded vocab, BN = 256)
  const void* ce_tgt;      // targets (int64 if ce_tgt_i64 else int32), row m = b * ce_T + t
  int ce_tgt_i64, ce_T;
  long long ce_tgt_ld;
  const float* ce_roww;    // per-row loss weight or null
  int ce_V;                // real classes (columns >= V are padding)
  float ce_S;              // softcap
  float* ce_part;          // [M][2 * tiles_n] partial sums of exp(y - S)
  float* ce_yc;            // [M] target's capped logit
  float* ce_loss;          // [M] w * (S + log(sum) - y_c), 0 for ignored targets
  int ce_write_dz;         // store z and rewrite it as dz
  TpArgs tp;
};

// PAIR: the tile is computed by a 2-CTA cluster (tcgen05 cta_group::2): 256 rows x BN,
// each CTA holding 128 rows of A and BN / 2 rows of B per stage, so per CTA a stage is
// 32 KB and six fit.
template <int BN, bool PAIR = false>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int BNH = PAIR ? BN / 2 : BN;  // rows of B this CTA loads per stage
  static constexpr int STAGES = PAIR ? 6 : (BN == 256) ? 4 : 6;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BNH * BK * 2;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int QSLOTS = 4;  // tile-id ring
  static constexpr size_t SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + (2 * STAGES + 5 + 2 * QSLOTS) * 8 + 64;
  static constexpr size_t SMEM_ALL = SMEM + 1024 + 8 * 4096;  // + epilogue staging tiles
};

template <int MODE>
__device__ __forceinline__ void decode_tile(int t, const GemmArgs& a, int& mb, int& nb, int& ks, int& bi) {
  if constexpr (MODE != MODE_PLAIN) {
    // m-major raster in rank order: AG starts at this rank's rows, RS at the next rank's
    // (own rows last); no split-K, no batch.
    const int mr = a.tp.rows_per_rank >> 7;
    const int first = MODE == MODE_AG ? a.tp.rank : (a.tp.rank + 1) % a.tp.world;
    const int m0 = t / a.tiles_n;
    nb = t - m0 * a.tiles_n;
    mb = (m0 + first * mr) % a.tiles_m;
    ks = 0;
    bi = 0;
    return;
  }
  const int per_split = a.tiles_m * a.tiles_n;
  const int per_batch = per_split * a.split_k;
  bi = t / per_batch;
  t -= bi * per_batch;
  ks = t / per_split;
  const int r = t - ks * per_split;
  constexpr int GROUP = 8;
  const int group_size = GROUP * a.tiles_n;
  const int g = r / group_size;
  const int first_m = g * GROUP;
  const int gm = min(GROUP, a.tiles_m - first_m);
  const int rr = r - g * group_size;
  mb = first_m + rr % gm;
  nb = rr / gm;
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu_u32(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Bounded wait until *flag has reached `epoch` (wrap-safe).  sys scope for words written
// by peers, gpu scope for words written by other CTAs of this kernel.
template <bool SYS>
__device__ __forceinline__ bool wait_epoch(const uint32_t* flag, uint32_t epoch, volatile int* abort_flag, int* err,
                                           int code) {
  const unsigned long long t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    const uint32_t v = SYS ? ld_acquire_sys_u32(flag) : ld_acquire_gpu_u32(flag);
    if ((int)(v - epoch) >= 0) return true;
    if ((++it & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        *abort_flag = 1;
        if (err) atomicOr(err, code);
        return false;
      }
    }
  }
}

// Split-K finish of one warp's region (32 rows x half the tile's columns): counts the
// splits that have added into it; the last one converts the fp32 sums to the bf16 output
// (optionally + residual or relu^2) and zeroes the workspace and the counter, so the next
// launch starts clean without a memset (CUDA-graph friendly decode GEMMs).
template <int BN>
__device__ __noinline__ void split_finish(const GemmArgs& a, int mb, int nb, int bi, int q, int hf, int warp, int lane) {
  __threadfence();  // this lane's partial-sum atomics are visible before the count moves
  __syncwarp();
  int last = 0;
  const long long slot = (((long long)bi * a.tiles_m + mb) * a.tiles_n + nb) * 8 + (warp - 2);
  if (lane == 0) last = atomicAdd(a.fin_cnt + slot, 1) == a.split_k - 1;
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  __threadfence();
  const int row = mb * 128 + q * 32 + lane;
  if (row < a.M) {
    float* ws = reinterpret_cast<float*>(a.D) + bi * a.d_bstride + (long long)row * a.ldd;
    __nv_bfloat16* out = a.fin_out + (long long)row * a.ld_fin;
    for (int c = hf * (BN / 64); c < (hf + 1) * (BN / 64); ++c) {
      const int col0 = nb * BN + c * 32;
      if (col0 >= a.N) break;
      float v[32];
      if (col0 + 32 <= a.N) {
        // whole chunk: every load is issued before any store (one memory round trip)
        float4 w4[8];
        uint4 r4[4];
#pragma unroll
        for (int i = 0; i < 8; ++i) w4[i] = __ldcg(reinterpret_cast<const float4*>(ws + col0) + i);
        if (a.R != nullptr) {
#pragma unroll
          for (int i = 0; i < 4; ++i) r4[i] = *reinterpret_cast<const uint4*>(a.R + (long long)row * a.ldr + col0 + 8 * i);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[4 * i] = w4[i].x; v[4 * i + 1] = w4[i].y; v[4 * i + 2] = w4[i].z; v[4 * i + 3] = w4[i].w;
        }
        if (a.R != nullptr) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&r4[i]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(h2[j]);
              v[8 * i + 2 * j] += a.rcoef * f.x;
              v[8 * i + 2 * j + 1] += a.rcoef * f.y;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (a.fin_relu2) {
            const float h = __bfloat162float(__float2bfloat16_rn(v[i])) - a.tau;
            v[i] = h > 0.f ? h * h : 0.f;
          }
        }
        uint4 ov[4];
        uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
        for (int i = 0; i < 16; ++i) ow[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
        for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(out + col0)[i] = ov[i];
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<float4*>(ws + col0)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        const int n = a.N - col0;
        for (int i = 0; i < n; ++i) {
          float x = __ldcg(ws + col0 + i);
          if (a.R != nullptr) x += a.rcoef * __bfloat162float(a.R[(long long)row * a.ldr + col0 + i]);
          if (a.fin_relu2) {
            const float h = __bfloat162float(__float2bfloat16_rn(x)) - a.tau;
            x = h > 0.f ? h * h : 0.f;
          }
          out[col0 + i] = __float2bfloat16_rn(x);
          ws[col0 + i] = 0.f;
        }
      }
    }
  }
  __syncwarp();
  if (lane == 0) a.fin_cnt[slot] = 0;
}

template <int MODE>
struct ModeThreads {
  static constexpr int value = MODE == MODE_AG ? 384 : 320;
};

template <int BN, bool A_MN, bool B_MN, int EPI, int MODE, bool PAIR = false>
__global__ void __launch_bounds__(ModeThreads<MODE>::value, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmD2,
                     const __grid_constant__ GemmArgs args) {
  static_assert(!PAIR || (MODE == MODE_PLAIN && BN == 256), "CTA pairs: plain GEMMs with 256-wide tiles");
  using C = GemmCfg<BN, PAIR>;
  constexpr int BM = C::BM, BK = C::BK, STAGES = C::STAGES, QS = C::QSLOTS, BNH = C::BNH;
  constexpr uint32_t IDESC = umma_idesc_bf16(PAIR ? 2 * BM : BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * C::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* qfull = drain + 1;
  uint64_t* qempty = qfull + QS;
  int* qtile = reinterpret_cast<int*>(qempty + QS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qtile + QS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* copy_word = reinterpret_cast<volatile int*>(tmem_slot + 2);
  // per-epilogue-warp staging tile [32 rows][64 cols] bf16 (4 KB each, 8 warps), 1 KB
  // aligned: the 128-byte-swizzled layout TMA stores read
  uint8_t* staging = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tmem_slot + 4) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pair: rank 0 (the leader) issues the MMAs for both; its full[] barriers count
  // both CTAs' TMA bytes and its tempty[] barriers both CTAs' epilogue warps.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = crank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], PAIR ? 16 : 256);  // pair: lane 0 of the 8 epilogue warps of each CTA
    }
    for (int i = 0; i < QS; ++i) {
      mbar_init(&qfull[i], 1);
      // MMA thread (the pair's leader only) + one lane of each epilogue warp
      mbar_init(&qempty[i], (PAIR && !leader) ? 8 : 9);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C::TMEM_COLS);  // the same warp of both CTAs
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // barrier inits visible to the peer before any remote arrive
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer + tile source
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int qs = 0;
      uint32_t qph = 0;
      bool ok = true;
      uint32_t out_valid = 0, out_parity = 0;  // per-stage: a load is in flight / its phase parity
      int ready_mb = -1;
      int static_t = PAIR ? (int)cluster_id_x() : (int)blockIdx.x;
      const int t_stride = PAIR ? (int)nclusters_x() : (int)gridDim.x;
      while (ok) {
        int t;
        if constexpr (MODE == MODE_PLAIN) {
          t = static_t;
          static_t += t_stride;
        } else {
          t = (int)atomicAdd(args.tp.sched, 1u);
        }
        if (t >= args.num_tiles) t = -1;
        if (!mbar_wait(&qempty[qs], qph ^ 1u, abort_flag, args.err, ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        qtile[qs] = t;
        mbar_arrive(&qfull[qs]);
        if (++qs == QS) {
          qs = 0;
          qph ^= 1u;
        }
        if (t < 0) break;
        int mb, nb, ks, bi;
        decode_tile<MODE>(t, args, mb, nb, ks, bi);
        if constexpr (PAIR) mb = 2 * mb + (int)crank;  // this CTA's 128-row half of the pair tile
        if constexpr (MODE == MODE_AG) {
          if (mb / (args.tp.rows_per_rank >> 7) != args.tp.rank && mb != ready_mb) {
            if (!wait_epoch<false>(args.tp.ag_done + mb, args.tp.epoch, abort_flag, args.err, ERR_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();  // generic-proxy copies -> this thread's TMA reads
            ready_mb = mb;
          }
        }
        const int kb0 = ks * args.kb_per_split;
        const int kb1 = min(kb0 + args.kb_per_split, args.kb_total);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.err, ERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
          if constexpr (PAIR) {
            // Each CTA loads its own halves into its own shared memory; the leader's full[]
            // barrier counts the bytes of both.
            if (leader) {
              mbar_arrive_expect_tx(&full[stage], 2 * (C::A_BYTES + C::B_BYTES));
              out_valid |= 1u << stage;
              out_parity = (out_parity & ~(1u << stage)) | (phase << stage);
            }
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            if (!A_MN) {
              tma_load_3d_pair(a_dst, &tmA, fb, kb * BK, mb * BM, bi);
            } else {
#pragma unroll
              for (int p = 0; p < BM / 64; ++p) tma_load_3d_pair(a_dst + p * 8192, &tmA, fb, mb * BM + p * 64, kb * BK, bi);
            }
            const int n0 = nb * BN + (int)crank * BNH;
            if (!B_MN) {
              tma_load_3d_pair(b_dst, &tmB, fb, kb * BK, n0, bi);
            } else {
#pragma unroll
              for (int p = 0; p < BNH / 64; ++p) tma_load_3d_pair(b_dst + p * 8192, &tmB, fb, n0 + p * 64, kb * BK, bi);
            }
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES + C::B_BYTES);
          out_valid |= 1u << stage;
          out_parity = (out_parity & ~(1u << stage)) | (phase << stage);
          if (!A_MN) {
            tma_load_3d(a_dst, &tmA, &full[stage], kb * BK, mb * BM, bi);
          } else {
#pragma unroll
            for (int p = 0; p < BM / 64; ++p) tma_load_3d(a_dst + p * 8192, &tmA, &full[stage], mb * BM + p * 64, kb * BK, bi);
          }
          if (!B_MN) {
            tma_load_3d(b_dst, &tmB, &full[stage], kb * BK, nb * BN, bi);
          } else {
#pragma unroll
            for (int p = 0; p < BN / 64; ++p) tma_load_3d(b_dst + p * 8192, &tmB, &full[stage], nb * BN + p * 64, kb * BK, bi);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        if constexpr (PAIR) {
          // This CTA's loads complete on the leader's barriers, which it cannot wait on:
          // give any copy still in flight a bounded moment to land before the CTA exits.
          const unsigned long long t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 5000000ull) {
          }
        }
        // Drain: wait (bounded) until every load issued into a stage has landed, so no
        // bulk copy is still writing shared memory when the CTA exits.
        for (int s = 0; s < STAGES; ++s) {
          if (!((out_valid >> s) & 1u)) continue;
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], (out_parity >> s) & 1u)) {
            if (globaltimer_ns() - t0 > 100000000ull) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      int qs = 0;
      uint32_t qph = 0;
      bool ok = true;
      while (ok) {
        if (!mbar_wait(&qfull[qs], qph, abort_flag, args.err, ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        const int t = qtile[qs];
        mbar_arrive(&qempty[qs]);
        if (++qs == QS) {
          qs = 0;
          qph ^= 1u;
        }
        if (t < 0) break;
        int mb, nb, ks, bi;
        decode_tile<MODE>(t, args, mb, nb, ks, bi);
        const int kb0 = ks * args.kb_per_split;
        const int kb1 = min(kb0 + args.kb_per_split, args.kb_total);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, args.err, ERR_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.err, ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc, bdesc;
            if (!A_MN) adesc = umma_desc_sw128(a_addr + kk * 32, 16, 1024);
            else adesc = umma_desc_sw128(a_addr + kk * 2048, 8192, 1024);
            if (!B_MN) bdesc = umma_desc_sw128(b_addr + kk * 32, 16, 1024);
            else bdesc = umma_desc_sw128(b_addr + kk * 2048, 8192, 1024);
            if constexpr (PAIR) umma_bf16_pair(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            else umma_bf16(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          // stage is free (in both CTAs of a pair) once these MMAs have read it
          if constexpr (PAIR) {
            umma_commit_pair(smem_u32(&empty[stage]));
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          } else {
            umma_commit(&empty[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // accumulator ready for the epilogue (of both CTAs of a pair)
        if constexpr (PAIR) {
          umma_commit_pair(smem_u32(&tfull[acc]));
          umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
        } else {
          umma_commit(&tfull[acc]);
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        // Let every MMA already issued finish before TMEM is released.
        if constexpr (PAIR) umma_commit_pair(smem_u32(drain));
        else umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (globaltimer_ns() - t0 > 100000000ull) break;
        }
      }
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int hf = (warp - 2) >> 2;  // column half of the tile this warp drains
    const float alpha = args.alpha * (args.alpha_ptr ? *args.alpha_ptr : 1.f);
    int acc = 0;
    uint32_t acc_phase = 0;
    int qs = 0;
    uint32_t qph = 0;
    // Hand accumulator a back to the MMA issuer (after tc_fence_before): every thread of a
    // single CTA, or lane 0 of each warp of both CTAs on the pair leader's barrier.
    auto release_acc = [&](int a_) {
      if constexpr (PAIR) {
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&tempty[a_]);
          else mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[a_]), 0));
        }
      } else {
        mbar_arrive(&tempty[a_]);
      }
    };
    while (true) {
      if (!mbar_wait_warp(&qfull[qs], qph, abort_flag, args.err, ERR_TIMEOUT_EPILOGUE)) break;
      const int t = qtile[qs];
      __syncwarp();
      if (lane == 0) mbar_arrive(&qempty[qs]);
      if (++qs == QS) {
        qs = 0;
        qph ^= 1u;
      }
      if (t < 0) break;
      int mb, nb, ks, bi;
      decode_tile<MODE>(t, args, mb, nb, ks, bi);
      if constexpr (PAIR) mb = 2 * mb + (int)crank;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, args.err, ERR_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      if constexpr (MODE == MODE_RS) {
        // ---- reduce-scatter epilogue
        const int mr = args.tp.rows_per_rank >> 7;
        const int owner = mb / mr;
        const int lrow = row - owner * args.tp.rows_per_rank;
        const int tiles_per_rank = mr * args.tiles_n;
        const int tile_local = (mb - owner * mr) * args.tiles_n + nb;
        const int rank = args.tp.rank;
        const long long N = args.N;
        bool wait_ok = true;
        if (owner == rank) {
          for (int s = 0; s < args.tp.world && wait_ok; ++s) {
            if (s == rank) continue;
            const uint32_t* f = args.tp.rs_flag[rank] + ((long long)s * tiles_per_rank + tile_local) * 8 + hf * 4 + q;
            wait_ok = wait_epoch<true>(f, args.tp.epoch, abort_flag, args.err, ERR_TIMEOUT_PEER);
          }
          wait_ok = __all_sync(0xffffffffu, wait_ok) != 0;
        }
        if (!wait_ok) break;
        if (owner != rank) {
          // Peer rows: bf16 partials to the owner's receive buffer.  Each 64-column slab is
          // staged in this warp's swizzled smem tile (thread = row), then written out as
          // whole 128-byte row segments, four rows per instruction.
          uint8_t* stg = staging + (warp - 2) * 4096;
          __nv_bfloat16* dst_base = args.tp.rs_recv[owner] + (long long)rank * args.tp.rows_per_rank * N;
#pragma unroll 1
          for (int c2 = hf * (BN / 128); c2 < (hf + 1) * (BN / 128); ++c2) {
            uint32_t r0[32], r1[32];
            __syncwarp();
            tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + c2 * 64), r0);
            tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + c2 * 64 + 32), r1);
            tmem_ld_wait();
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              const uint32_t* src = cc < 4 ? r0 + cc * 8 : r1 + (cc - 4) * 8;
              uint4 u;
              u.x = pack_bf16x2(__uint_as_float(src[0]) * alpha, __uint_as_float(src[1]) * alpha);
              u.y = pack_bf16x2(__uint_as_float(src[2]) * alpha, __uint_as_float(src[3]) * alpha);
              u.z = pack_bf16x2(__uint_as_float(src[4]) * alpha, __uint_as_float(src[5]) * alpha);
              u.w = pack_bf16x2(__uint_as_float(src[6]) * alpha, __uint_as_float(src[7]) * alpha);
              *reinterpret_cast<uint4*>(stg + lane * 128 + ((cc ^ (lane & 7)) << 4)) = u;
            }
            __syncwarp();
            const int col0 = nb * BN + c2 * 64;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = i * 4 + (lane >> 3), cc = lane & 7;
              const int gcol = col0 + cc * 8;
              const int lr = mb * BM + q * 32 + rr - owner * args.tp.rows_per_rank;
              if (gcol < args.N)
                *reinterpret_cast<uint4*>(dst_base + (long long)lr * N + gcol) =
                    *reinterpret_cast<const uint4*>(stg + rr * 128 + ((cc ^ (rr & 7)) << 4));
            }
          }
        } else {
#pragma unroll 1
        for (int c = hf * (BN / 64); c < (hf + 1) * (BN / 64); ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + c * 32), r);
          tmem_ld_wait();
          const int col0 = nb * BN + c * 32;
          if (col0 >= args.N) continue;
          const bool full_cols = col0 + 32 <= args.N;
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * alpha;
            for (int s = 0; s < args.tp.world; ++s) {
              if (s == rank) continue;
              const __nv_bfloat16* src = args.tp.rs_recv[rank] + ((long long)s * args.tp.rows_per_rank + lrow) * N + col0;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                if (col0 + 8 * i < args.N) {   // N % 8 == 0: whole 8-column groups
                  const uint4 x = __ldcg(reinterpret_cast<const uint4*>(src) + i);
                  const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float2 f = __bfloat1622float2(x2[j]);
                    v[8 * i + 2 * j] += f.x;
                    v[8 * i + 2 * j + 1] += f.y;
                  }
                }
              }
            }
            __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.D) + (long long)lrow * args.ldd + col0;
            if (args.R != nullptr) {
              const __nv_bfloat16* rr = args.R + (long long)lrow * args.ldr + col0;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (full_cols || col0 + i < args.N) v[i] += args.rcoef * __bfloat162float(rr[i]);
            }
            if (full_cols) {
              uint4 ov[4];
              uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
              for (int i = 0; i < 16; ++i) ow[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
              for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(out)[i] = ov[i];
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col0 + i < args.N) out[i] = __float2bfloat16_rn(v[i]);
            }
          }
        }
        tc_fence_before();
        release_acc(acc);
        if (owner != rank) {
          // This lane quarter of the tile is in the owner's receive buffer: announce it.  The
          // warp barrier orders every lane's stores before lane 0's system-scope release
          // (cumulative), so one release per warp replaces a fence per thread.
          __syncwarp();
          if (lane == 0)
            st_release_sys_u32(args.tp.rs_flag[owner] + ((long long)rank * tiles_per_rank + tile_local) * 8 + hf * 4 + q,
                               args.tp.epoch);
        }
      } else if (EPI == EPI_F32 && args.tma_store) {
        // ---- fp32 output through TMA: 32 rows x 32 columns staged per warp (128-byte
        // swizzle); accumulation (beta = 1 or split-K) is a bulk reduce-add in L2, a plain
        // result a bulk store -- no per-thread read-modify-write or atomics.
        uint8_t* stg = staging + (warp - 2) * 4096;
        const int row0 = mb * BM + q * 32;
        const bool reduce = args.split_k > 1 || args.beta != 0.f;
#pragma unroll 1
        for (int c = hf * (BN / 64); c < (hf + 1) * (BN / 64); ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + c * 32), r);
          tmem_ld_wait();
          const int col0 = nb * BN + c * 32;
          if (col0 >= args.N) continue;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_float4(__uint_as_float(r[4 * j]) * alpha, __uint_as_float(r[4 * j + 1]) * alpha,
                            __uint_as_float(r[4 * j + 2]) * alpha, __uint_as_float(r[4 * j + 3]) * alpha);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < args.M) {
            if (reduce) tma_reduce_add_3d(&tmD, stg, col0, row0, bi);
            else tma_store_3d(&tmD, stg, col0, row0, bi);
            bulk_commit_group();
            bulk_wait_group_read<0>();
          }
          __syncwarp();
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
        tc_fence_before();
        release_acc(acc);
      } else if (EPI != EPI_F32 && args.tma_store) {
        // ---- bf16 outputs through TMA stores: each warp stages its 32 rows x 64 columns
        // (128-byte swizzle) and one lane stores the slab, so global writes are whole lines
        // instead of 32 rows touched per store instruction.
        uint8_t* stg = staging + (warp - 2) * 4096;
        const int row0 = mb * BM + q * 32;
        const bool row_ok = row < args.M;
        auto stage = [&](const float* v) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            uint4 u;
            u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
            u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
            u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
            u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
            *reinterpret_cast<uint4*>(stg + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
          }
          fence_proxy_async_smem();
          __syncwarp();
        };
        auto store = [&](const CUtensorMap* map, int col0) {
          if (lane == 0 && row0 < args.M) {  // rows past M are clipped by TMA; skip all-outside slabs
            tma_store_3d(map, stg, col0, row0, bi);
            bulk_commit_group();
            bulk_wait_group_read<0>();  // the slab may be overwritten after this
          }
          __syncwarp();
        };
        bool roped = false;
        // EPI_CE: this thread's row target and its running partial sum over the tile half
        long long ce_cls = -1;
        float ce_sum = 0.f;
        if constexpr (EPI == EPI_CE) {
          if (row_ok) {
            const long long ti = (long long)(row / args.ce_T) * args.ce_tgt_ld + row % args.ce_T;
            ce_cls = args.ce_tgt_i64 ? reinterpret_cast<const long long*>(args.ce_tgt)[ti]
                                     : (long long)reinterpret_cast<const int*>(args.ce_tgt)[ti];
          }
        }
        if constexpr (EPI == EPI_ROPE && MODE == MODE_PLAIN && BN == 256) {
          const int hcol = nb * BN + hf * 128;  // first column of this warp's head
          if (hcol < args.rope_cols) {
            // ---- RoPE + RMSNorm of one 128-wide head per thread-row.  x = bf16(acc) (the
            // value a separate pass would read back), y1 = x1 c + x2 s, y2 = x2 c - x1 s over
            // the two 64-column halves, out = y / rms(y).  Pass 1 sums y^2; passes 2 and 3
            // recompute y1 and y2 from TMEM (cheap re-reads instead of 128 live registers)
            // and store them as two staged 64-column slabs.
            roped = true;
            const int pos = (row_ok ? row : 0) % args.rope_T;
            const __nv_bfloat16* crow = args.rope_cos + (long long)pos * 64;
            const __nv_bfloat16* srow = args.rope_sin + (long long)pos * 64;
            const uint32_t tb = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + hf * 128);
            // f(k, y1, y2) for the rotated pair at half-column 32p + k, k < 32
            auto rot = [&](int p, auto&& f) {
              uint32_t ra[32], rb[32];
              __syncwarp();
              tmem_ld_32x32b_x32(tb + p * 32, ra);
              tmem_ld_32x32b_x32(tb + 64 + p * 32, rb);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 cu = reinterpret_cast<const uint4*>(crow + p * 32)[i];
                const uint4 su = reinterpret_cast<const uint4*>(srow + p * 32)[i];
                const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&cu);
                const __nv_bfloat162* s2v = reinterpret_cast<const __nv_bfloat162*>(&su);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 cf = __bfloat1622float2(c2[j]), sf = __bfloat1622float2(s2v[j]);
#pragma unroll
                  for (int e = 0; e < 2; ++e) {
                    const int k = 8 * i + 2 * j + e;
                    const float c = e ? cf.y : cf.x, sn = e ? sf.y : sf.x;
                    const float x1 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(ra[k]) * alpha));
                    const float x2 = __bfloat162float(__float2bfloat16_rn(__uint_as_float(rb[k]) * alpha));
                    f(k, x1 * c + x2 * sn, x2 * c - x1 * sn);
                  }
                }
              }
            };
            float ss = 0.f;
#pragma unroll 1
            for (int p = 0; p < 2; ++p)
              rot(p, [&](int, float y1, float y2) { ss += y1 * y1 + y2 * y2; });
            const float rn = rsqrtf(ss * (1.f / 128.f) + 1.1920928955078125e-07f);
            if (row_ok && args.rope_rstd != nullptr)
              args.rope_rstd[(long long)row * args.rope_heads + hcol / 128] = rn;
#pragma unroll 1
            for (int which = 0; which < 2; ++which) {
#pragma unroll 1
              for (int p = 0; p < 2; ++p) {  // 32 columns at a time into the swizzled slab
                float v[32];
                rot(p, [&](int k, float y1, float y2) { v[k] = (which ? y2 : y1) * rn; });
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  uint4 u;
                  u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
                  u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
                  u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
                  u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
                  *reinterpret_cast<uint4*>(stg + lane * 128 + (((4 * p + j) ^ (lane & 7)) << 4)) = u;
                }
              }
              fence_proxy_async_smem();
              __syncwarp();
              store(&tmD, hcol + which * 64);
            }
          }
        }
#pragma unroll 1
        for (int s2 = hf * (BN / 128); s2 < (hf + 1) * (BN / 128) && !roped; ++s2) {
          uint32_t r0[32], r1[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + s2 * 64), r0);
          tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + s2 * 64 + 32), r1);
          tmem_ld_wait();
          const int col0 = nb * BN + s2 * 64;
          if (col0 >= args.N) continue;
          float v[64];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            v[i] = __uint_as_float(r0[i]) * alpha;
            v[32 + i] = __uint_as_float(r1[i]) * alpha;
          }
          if constexpr (EPI == EPI_BF16) {
            if (args.R != nullptr && row_ok) {
              const __nv_bfloat16* rr = args.R + bi * args.r_bstride + (long long)row * args.ldr + col0;
              const float rc = args.rcoef;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                if (col0 + 8 * i < args.N) {  // N % 8 == 0 on this path
                  const uint4 u = reinterpret_cast<const uint4*>(rr)[i];
                  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float2 f = __bfloat1622float2(h2[j]);
                    v[8 * i + 2 * j] += rc * f.x;
                    v[8 * i + 2 * j + 1] += rc * f.y;
                  }
                }
              }
            }
          } else if constexpr (EPI == EPI_RELU2) {
            stage(v);                      // pre-activation h
            store(&tmD2, col0);
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              const float h = __bfloat162float(__float2bfloat16_rn(v[i])) - args.tau;
              const float rl = h > 0.f ? h : 0.f;
              v[i] = rl * rl;
            }
          } else if constexpr (EPI == EPI_RELU2_BWD) {
            float hf8[64];
            if (row_ok) {
              const __nv_bfloat16* hh = args.R + bi * args.r_bstride + (long long)row * args.ldr + col0;
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                uint4 u = make_uint4(0u, 0u, 0u, 0u);
                if (col0 + 8 * i < args.N) u = reinterpret_cast<const uint4*>(hh)[i];
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 f = __bfloat1622float2(h2[j]);
                  hf8[8 * i + 2 * j] = f.x;
                  hf8[8 * i + 2 * j + 1] = f.y;
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 64; ++i) hf8[i] = 0.f;
            }
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              const float g = __bfloat162float(__float2bfloat16_rn(v[i]));
              const float h = hf8[i] - args.tau;
              v[i] = h > 0.f ? g * (2.f * h) : 0.f;
            }
          } else if constexpr (EPI == EPI_CE) {
            const float S = args.ce_S, invS = 1.f / S;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              const float z = __bfloat162float(__float2bfloat16_rn(v[i]));
              const int j = col0 + i;
              if (j < args.ce_V) {
                const float y = S * tanhf(z * invS);
                ce_sum += __expf(y - S);
                if (j == ce_cls) args.ce_yc[row] = y;
              }
            }
            if (!args.ce_write_dz) continue;
          }
          stage(v);
          store(&tmD, col0);
        }
        if constexpr (EPI == EPI_CE) {
          if (row_ok) args.ce_part[(long long)row * (2 * args.tiles_n) + nb * 2 + hf] = ce_sum;
        }
        if (lane == 0) bulk_wait_group<0>();
        __syncwarp();
        tc_fence_before();
        release_acc(acc);

      } else {
        const bool row_ok = row < args.M;
#pragma unroll 1
        for (int c = hf * (BN / 64); c < (hf + 1) * (BN / 64); ++c) {
          uint32_t r[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * BN + c * 32), r);
          tmem_ld_wait();
          const int col0 = nb * BN + c * 32;
          if (!row_ok || col0 >= args.N) continue;
          const bool full_cols = col0 + 32 <= args.N;
          float v[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * alpha;
        if constexpr (EPI == EPI_F32) {
          float* out = reinterpret_cast<float*>(args.D) + bi * args.d_bstride + (long long)row * args.ldd + col0;
          if (full_cols) {
            float4* o4 = reinterpret_cast<float4*>(out);
            if (args.split_k > 1) {
#pragma unroll
              for (int i = 0; i < 8; ++i) atomicAdd(o4 + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
            } else if (args.beta != 0.f) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float4 o = o4[i];
                o.x += v[4 * i]; o.y += v[4 * i + 1]; o.z += v[4 * i + 2]; o.w += v[4 * i + 3];
                o4[i] = o;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (col0 + i < args.N) {
                if (args.split_k > 1) atomicAdd(out + i, v[i]);
                else out[i] = v[i] + (args.beta != 0.f ? out[i] : 0.f);
              }
            }
          }
        } else {
          __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.D) + bi * args.d_bstride + (long long)row * args.ldd + col0;
          if constexpr (EPI == EPI_BF16) {
            if (args.R != nullptr) {
              const __nv_bfloat16* rr = args.R + bi * args.r_bstride + (long long)row * args.ldr + col0;
              const float rc = args.rcoef;
              if (full_cols) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  uint4 u = reinterpret_cast<const uint4*>(rr)[i];
                  const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    float2 f = __bfloat1622float2(h2[j]);
                    v[8 * i + 2 * j] += rc * f.x;
                    v[8 * i + 2 * j + 1] += rc * f.y;
                  }
                }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (col0 + i < args.N) v[i] += rc * __bfloat162float(rr[i]);
              }
            }
          } else if constexpr (EPI == EPI_RELU2) {
            __nv_bfloat16* hout = reinterpret_cast<__nv_bfloat16*>(args.D2) + bi * args.d2_bstride + (long long)row * args.ldd2 + col0;
            if (full_cols) {
              uint4 hv[4];
              uint32_t* hw = reinterpret_cast<uint32_t*>(hv);
#pragma unroll
              for (int i = 0; i < 16; ++i) hw[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
              for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(hout)[i] = hv[i];
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col0 + i < args.N) hout[i] = __float2bfloat16_rn(v[i]);
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float h = __bfloat162float(__float2bfloat16_rn(v[i])) - args.tau;
              const float rl = h > 0.f ? h : 0.f;
              v[i] = rl * rl;
            }
          } else if constexpr (EPI == EPI_RELU2_BWD) {
            const __nv_bfloat16* hh = args.R + bi * args.r_bstride + (long long)row * args.ldr + col0;
            float hf[32];
            if (full_cols) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                uint4 u = reinterpret_cast<const uint4*>(hh)[i];
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  float2 f = __bfloat1622float2(h2[j]);
                  hf[8 * i + 2 * j] = f.x;
                  hf[8 * i + 2 * j + 1] = f.y;
                }
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) hf[i] = (col0 + i < args.N) ? __bfloat162float(hh[i]) : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float g = __bfloat162float(__float2bfloat16_rn(v[i]));
              const float h = hf[i] - args.tau;
              v[i] = h > 0.f ? g * (2.f * h) : 0.f;
            }
          }
          if (full_cols) {
            uint4 ov[4];
            uint32_t* ow = reinterpret_cast<uint32_t*>(ov);
#pragma unroll
            for (int i = 0; i < 16; ++i) ow[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
#pragma unroll
            for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(out)[i] = ov[i];
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < args.N) out[i] = __float2bfloat16_rn(v[i]);
          }
        }
      }

        tc_fence_before();
        release_acc(acc);
        if constexpr (EPI == EPI_F32) {
          if (args.fin_out != nullptr) split_finish<BN>(args, mb, nb, bi, q, hf, warp, lane);
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  } else if constexpr (MODE == MODE_AG) {
    // ------------------------------------------------------------ all-gather copy warps (6, 7)
    const int ct = threadIdx.x - 320;  // 0..63
    const TpArgs& tp = args.tp;
    if (ct < tp.world && ct != tp.rank) {
      // this rank's rows of this call are in its gather buffer (written by earlier kernels)
      __threadfence_system();
      st_release_sys_u32(tp.ag_ready[ct] + tp.rank, tp.epoch);
    }
    const int mr = tp.rows_per_rank >> 7;
    const int jobs = (tp.world - 1) * mr;
    const int start = (int)((long long)blockIdx.x * jobs / gridDim.x);
    const int vpr = tp.ag_row_bytes >> 4;  // 16-byte vectors per row
    const int total = BM * vpr;
    uint32_t ready_mask = 1u << tp.rank;
    for (int i = 0; i < jobs; ++i) {
      const int j = (start + i) % jobs;
      const int gmb = ((tp.rank + 1) * mr + j) % args.tiles_m;
      const int owner = gmb / mr;
      if (ct == 0) {
        int st = 0;  // 0 skip, 1 copy, 2 abort
        if (*abort_flag) {
          st = 2;
        } else if (atomicMax(tp.ag_claim + j, tp.epoch) != tp.epoch) {
          st = 1;
          if (!((ready_mask >> owner) & 1u)) {
            if (wait_epoch<true>(tp.ag_ready[tp.rank] + owner, tp.epoch, abort_flag, args.err, ERR_TIMEOUT_PEER))
              ready_mask |= 1u << owner;
            else
              st = 2;
          }
        }
        *copy_word = st;
      }
      named_bar_sync(2, 64);
      const int st = *copy_word;
      named_bar_sync(2, 64);
      if (st == 2) break;
      if (st == 0) continue;
      const uint8_t* src = tp.ag_src[owner] + (long long)gmb * BM * tp.ag_ld_bytes;
      uint8_t* dst = tp.ag_dst + (long long)gmb * BM * tp.ag_ld_bytes;
      for (int base = ct; base < total; base += 64 * 8) {
        uint4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int idx = base + u * 64;
          if (idx < total) {
            const int rr = idx / vpr, cc = idx - rr * vpr;
            v[u] = __ldcg(reinterpret_cast<const uint4*>(src + (long long)rr * tp.ag_ld_bytes) + cc);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int idx = base + u * 64;
          if (idx < total) {
            const int rr = idx / vpr, cc = idx - rr * vpr;
            reinterpret_cast<uint4*>(dst + (long long)rr * tp.ag_ld_bytes)[cc] = v[u];
          }
        }
      }
      fence_proxy_async_global();
      __threadfence();
      named_bar_sync(2, 64);
      if (ct == 0) st_release_gpu_u32(tp.ag_done + gmb, tp.epoch);
    }
  }

  tc_fence_before();
  // A pair's CTAs read each other's shared memory and arrive on each other's barriers:
  // neither may exit (or free TMEM) before both are done.
  if constexpr (PAIR) cluster_sync();
  else __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if constexpr (MODE != MODE_PLAIN) {
    if (threadIdx.x == 0) {
      // the last CTA to finish rewinds the tile counter for the next launch
      __threadfence();
      if (atomicAdd(args.tp.sched + 1, 1u) == gridDim.x - 1) {
        atomicExch(args.tp.sched, 0u);
        atomicExch(args.tp.sched + 1, 0u);
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    C10_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(p != nullptr && q == cudaDriverEntryPointSuccess, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// cuTensorMapEncodeTiled is a driver call and runs against whatever context is current on
// the calling thread.  The runtime makes a device's primary context current lazily, on the
// first runtime call of a thread that needs one, and the device guard skips cudaSetDevice
// when the requested index already equals the runtime's current one (0 on a fresh thread).
// So on a thread whose first CUDA work is a tensor-map encode -- PyTorch's autograd thread
// for device 0 when a backward pass starts in one of these ops -- no context is current
// yet, and the encode crashed the process there.  cudaSetDevice binds the primary context;
// it is issued once per thread and device (so never during a graph capture that follows
// warm-up calls).
static void bind_device_context() {
  thread_local int bound = -1;
  int dev = 0;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (bound != dev) {
    C10_CUDA_CHECK(cudaSetDevice(dev));
    bound = dev;
  }
}

// 2-D bf16 tensor map with 128-byte swizzle.  inner/outer are element extents,
// row_stride_elems the distance between consecutive outer indices.
CUtensorMap make_tmap_bf16(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                           uint32_t box_inner, uint32_t box_outer, uint64_t batch, uint64_t batch_stride_elems) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK(batch == 1 || (batch_stride_elems * 2) % 16 == 0, "TMA batch stride must be a multiple of 16 bytes");
  bind_device_context();
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {row_stride_elems * 2, (batch > 1 ? batch_stride_elems : row_stride_elems * outer) * 2};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", int(r));
  return m;
}

// fp32 variant (e.g. the destination of TMA bulk reduce-adds), 128-byte swizzle.
CUtensorMap make_tmap_f32(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                          uint32_t box_inner, uint32_t box_outer) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 4) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK(box_inner * 4 <= 128, "128-byte swizzle: inner box of at most 32 fp32");
  bind_device_context();
  CUtensorMap m;
  cuuint64_t dims[3] = {inner, outer, 1};
  cuuint64_t strides[2] = {row_stride_elems * 4, row_stride_elems * outer * 4};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (fp32) failed with code ", int(r));
  return m;
}

int num_sms(int dev) {
  static int cache[64] = {0};
  if (!cache[dev]) {
    cudaDeviceProp prop;
    C10_CUDA_CHECK(cudaGetDeviceProperties(&prop, dev));
    cache[dev] = prop.multiProcessorCount;
  }
  return cache[dev];
}

template <int BN, bool A_MN, bool B_MN, int EPI, int MODE = MODE_PLAIN, bool PAIR = false>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td, const CUtensorMap& td2,
                        const GemmArgs& a, int grid, cudaStream_t stream) {
  using C = GemmCfg<BN, PAIR>;
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, EPI, MODE, PAIR>;
  // every epilogue stages through the same per-warp tiles (TMA stores / reduce-adds, the
  // TP reduce-scatter)
  constexpr size_t smem = C::SMEM_ALL;
  static_assert(smem <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
  static bool attr_set = false;  // one per instantiation
  static int max_clusters = 0;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr_set = true;
  }
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(ModeThreads<MODE>::value, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (max_clusters == 0) {
      // Persistent grid: as many pairs as can be resident at once (GPCs need not hold an
      // even number of free SMs, so this can be below SMs / 2).
      cfg.gridDim = dim3(2 * 74, 1, 1);
      int n = 0;
      C10_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      max_clusters = n > 0 ? n : 1;
    }
    const int pairs = std::max(1, std::min(a.num_tiles, max_clusters));
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, td, td2, a));
    (void)grid;
    return;
  }
  kern<<<grid, ModeThreads<MODE>::value, smem, stream>>>(ta, tb, td, td2, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, bool PAIR = false>
static void dispatch(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                     const CUtensorMap& td, const CUtensorMap& td2, const GemmArgs& a, int grid, cudaStream_t s) {
#define TFB_CASE(AM, BM_, E) \
  if (a_mn == AM && b_mn == BM_ && epi == E) \
    return launch_gemm<BN, AM, BM_, E, MODE_PLAIN, PAIR>(ta, tb, td, td2, a, grid, s);
  TFB_CASE(false, false, EPI_BF16)
  TFB_CASE(false, false, EPI_RELU2)
  TFB_CASE(false, false, EPI_F32)
  TFB_CASE(false, true, EPI_BF16)
  TFB_CASE(false, true, EPI_RELU2_BWD)
  TFB_CASE(false, true, EPI_F32)
  TFB_CASE(true, true, EPI_F32)
  TFB_CASE(true, true, EPI_BF16)
  TFB_CASE(true, false, EPI_F32)
  TFB_CASE(true, false, EPI_BF16)
  if constexpr (BN == 256) {
    TFB_CASE(false, false, EPI_ROPE)
    TFB_CASE(false, false, EPI_CE)
  }
#undef TFB_CASE
  TORCH_CHECK(false, "unsupported gemm variant a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

template <int BN>
static void dispatch_tp(int mode, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                        const CUtensorMap& td, const CUtensorMap& td2, const GemmArgs& a, int grid, cudaStream_t s) {
#define TFB_TP(MD, BM_, E) \
  if (mode == MD && b_mn == BM_ && epi == E) return launch_gemm<BN, false, BM_, E, MD>(ta, tb, td, td2, a, grid, s);
  TFB_TP(MODE_AG, false, EPI_BF16)
  TFB_TP(MODE_AG, false, EPI_RELU2)
  TFB_TP(MODE_AG, true, EPI_BF16)
  TFB_TP(MODE_AG, true, EPI_RELU2_BWD)
  TFB_TP(MODE_RS, false, EPI_BF16)
  TFB_TP(MODE_RS, true, EPI_BF16)
#undef TFB_TP
  TORCH_CHECK(false, "unsupported tensor-parallel gemm variant mode=", mode, " b_mn=", b_mn, " epi=", epi);
}

// The TMA-store epilogue needs 16-byte aligned rows and whole 8-column groups.
static bool tma_store_ok(int64_t epi, int64_t N, const void* d, long long ldd, long long dbs, const void* d2,
                         long long ldd2, long long d2bs) {
  static const bool off = getenv("TFB_GEMM_NO_TMA_STORE") != nullptr;
  if (off || N % 8 != 0) return false;
  if (epi == EPI_F32)  // fp32: 16-byte rows, one batch (the tensor map is 2-D)
    return dbs == 0 && d != nullptr && (reinterpret_cast<uintptr_t>(d) & 15) == 0 && (ldd * 4) % 16 == 0;
  auto ok = [](const void* p, long long ld, long long bs) {
    return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * 2) % 16 == 0 && (bs * 2) % 16 == 0;
  };
  if (!ok(d, ldd, dbs)) return false;
  if (epi == EPI_RELU2 && !ok(d2, ldd2, d2bs)) return false;
  return true;
}

struct CeEpi {
  const void* tgt = nullptr;
  int tgt_i64 = 1, T = 1;
  long long tgt_ld = 0;
  const float* roww = nullptr;
  int V = 0;
  float S = 15.f;
  float* part = nullptr;
  float* yc = nullptr;
  float* loss = nullptr;
  int write_dz = 1;
};

// A: if !a_mn a [M, K] view (row stride lda), else a [K, M] view.  B likewise with N.
// Operands are 2-D, or 3-D with a leading batch dimension (all of A, B, D batched alike).
struct RopeEpi {
  const __nv_bfloat16* cos = nullptr;
  const __nv_bfloat16* sin = nullptr;
  int T = 0, cols = 0, heads = 0;
  float* rstd = nullptr;
};

static void gemm_bf16_impl(torch::Tensor A, bool a_mn, torch::Tensor B, bool b_mn, int64_t M, int64_t N, int64_t K,
                           torch::Tensor D, int64_t epi, double alpha, double beta, c10::optional<torch::Tensor> R,
                           c10::optional<torch::Tensor> D2, double tau, int64_t split_k, int64_t bn, torch::Tensor err,
                           c10::optional<torch::Tensor> alpha_t, double rcoef, const RopeEpi& rope,
                           const CeEpi& ce = CeEpi{}) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && D.is_cuda(), "gemm operands must be CUDA tensors");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm inputs must be bf16");
  const int64_t nb = A.dim() == 3 ? A.size(0) : 1;
  TORCH_CHECK(A.dim() == B.dim() && A.dim() == D.dim() && (A.dim() == 2 || A.dim() == 3), "operands must be 2-D or 3-D alike");
  if (A.dim() == 3) TORCH_CHECK(B.size(0) == nb && D.size(0) == nb, "batch sizes differ");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1 && D.stride(-1) == 1, "inner dimension must be contiguous");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "empty gemm");
  const int64_t a_bs = A.dim() == 3 ? A.stride(0) : 0, b_bs = B.dim() == 3 ? B.stride(0) : 0;
  if (A.dim() == 3) {
    A = A.select(0, 0); B = B.select(0, 0);
  }
  const int64_t d_bs = D.dim() == 3 ? D.stride(0) : 0;
  torch::Tensor Dfull = D;
  if (D.dim() == 3) D = D.select(0, 0);
  TORCH_CHECK(!a_mn ? (A.size(0) >= M && A.size(1) >= K) : (A.size(0) >= K && A.size(1) >= M), "A shape");
  TORCH_CHECK(!b_mn ? (B.size(0) >= N && B.size(1) >= K) : (B.size(0) >= K && B.size(1) >= N), "B shape");
  TORCH_CHECK(D.size(0) >= M && D.size(1) >= N, "D shape");
  const bool f32 = epi == EPI_F32;
  TORCH_CHECK(D.scalar_type() == (f32 ? at::kFloat : at::kBFloat16), "D dtype does not match epilogue");
  TORCH_CHECK(bn == 128 || bn == 256, "bn must be 128 or 256");
  c10::cuda::CUDAGuard guard(A.device());
  const int BM = 128, BK = 64;
  // 256-wide tiles over more than one 128-row block run on CTA pairs (tcgen05 cta_group::2:
  // 256 x 256 per pair, each CTA loading half of B), which halves the shared-memory /
  // L2 traffic of B per MMA; TFB_GEMM_PAIR=0 keeps one CTA per 128 x 256 tile.
  static const bool pair_on = getenv("TFB_GEMM_PAIR") == nullptr || getenv("TFB_GEMM_PAIR")[0] != '0';
  const bool pair = pair_on && bn == 256 && M > BM;
  const uint32_t b_rows = pair ? (uint32_t)bn / 2 : (uint32_t)bn;
  CUtensorMap ta = !a_mn ? make_tmap_bf16(A.data_ptr(), K, M, A.stride(0), 64, BM, nb, a_bs)
                         : make_tmap_bf16(A.data_ptr(), M, K, A.stride(0), 64, 64, nb, a_bs);
  CUtensorMap tb = !b_mn ? make_tmap_bf16(B.data_ptr(), K, N, B.stride(0), 64, b_rows, nb, b_bs)
                         : make_tmap_bf16(B.data_ptr(), N, K, B.stride(0), 64, 64, nb, b_bs);
  GemmArgs a{};
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  a.tiles_m = (int)((M + (pair ? 2 * BM : BM) - 1) / (pair ? 2 * BM : BM));
  a.tiles_n = (int)((N + bn - 1) / bn);
  a.kb_total = (int)((K + BK - 1) / BK);
  int sk = (int)std::max<int64_t>(1, std::min<int64_t>(split_k, a.kb_total));
  TORCH_CHECK(sk == 1 || f32, "split-K needs the fp32 accumulate epilogue");
  a.kb_per_split = (a.kb_total + sk - 1) / sk;
  sk = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;  // no empty splits
  a.split_k = sk;
  a.batch = (int)nb;
  a.num_tiles = a.tiles_m * a.tiles_n * sk * a.batch;
  if (sk > 1 && beta == 0.0) {
    if (Dfull.dim() == 3) Dfull.narrow(1, 0, M).narrow(2, 0, N).zero_();
    else D.narrow(0, 0, M).narrow(1, 0, N).zero_();
  }
  a.alpha = (float)alpha; a.beta = (float)beta; a.tau = (float)tau; a.rcoef = (float)rcoef;
  a.alpha_ptr = nullptr;
  if (alpha_t.has_value()) {
    TORCH_CHECK(alpha_t->scalar_type() == at::kFloat && alpha_t->is_cuda(), "alpha tensor must be CUDA fp32");
    a.alpha_ptr = alpha_t->data_ptr<float>();
  }
  a.D = D.data_ptr(); a.ldd = D.stride(0); a.d_bstride = d_bs;
  a.D2 = nullptr; a.ldd2 = 0; a.d2_bstride = 0; a.R = nullptr; a.ldr = 0; a.r_bstride = 0;
  if (epi == EPI_RELU2) {
    TORCH_CHECK(D2.has_value() && D2->scalar_type() == at::kBFloat16 && D2->stride(-1) == 1, "RELU2 needs D2");
    a.D2 = D2->data_ptr(); a.ldd2 = D2->stride(-2); a.d2_bstride = D2->dim() == 3 ? D2->stride(0) : 0;
  }
  if (R.has_value()) {
    TORCH_CHECK(R->scalar_type() == at::kBFloat16 && R->stride(-1) == 1, "R must be bf16 row-major");
    a.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()); a.ldr = R->stride(-2);
    a.r_bstride = R->dim() == 3 ? R->stride(0) : 0;
  }
  TORCH_CHECK(epi != EPI_RELU2_BWD || a.R != nullptr, "RELU2_BWD needs R = pre-activation");
  a.err = err.data_ptr<int>();
  CUtensorMap td = ta, td2 = ta;
  a.tma_store = tma_store_ok(epi, N, D.data_ptr(), a.ldd, d_bs, epi == EPI_RELU2 ? a.D2 : nullptr, a.ldd2, a.d2_bstride);
  if (a.tma_store && epi == EPI_F32) {
    if (nb != 1) a.tma_store = 0;
    else td = make_tmap_f32(a.D, N, M, a.ldd, 32, 32);
  } else if (a.tma_store) {
    td = make_tmap_bf16(a.D, N, M, a.ldd, 64, 32, nb, d_bs);
    if (epi == EPI_RELU2) td2 = make_tmap_bf16(a.D2, N, M, a.ldd2, 64, 32, nb, a.d2_bstride);
  }
  if (epi == EPI_CE) {
    TORCH_CHECK(a.tma_store && bn == 256 && !a_mn && !b_mn && nb == 1 && a.R == nullptr && ce.tgt != nullptr,
                "CE epilogue: 2-D K-major operands, bf16 TMA-store output, 256-wide tiles");
    a.ce_tgt = ce.tgt; a.ce_tgt_i64 = ce.tgt_i64; a.ce_T = ce.T; a.ce_tgt_ld = ce.tgt_ld; a.ce_roww = ce.roww;
    a.ce_V = ce.V; a.ce_S = ce.S; a.ce_part = ce.part; a.ce_yc = ce.yc; a.ce_loss = ce.loss;
    a.ce_write_dz = ce.write_dz;
  }
  a.rope_cos = rope.cos; a.rope_sin = rope.sin; a.rope_T = rope.T; a.rope_cols = rope.cols;
  a.rope_heads = rope.heads; a.rope_rstd = rope.rstd;
  if (epi == EPI_ROPE)
    TORCH_CHECK(rope.cos != nullptr && a.tma_store && bn == 256 && !a_mn && !b_mn && nb == 1 && a.R == nullptr,
                "RoPE epilogue: 2-D K-major operands, bf16 TMA-store output, 256-wide tiles, no residual");
  const int grid = std::min(a.num_tiles, num_sms(A.get_device()));
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (pair) dispatch<256, true>(a_mn, b_mn, (int)epi, ta, tb, td, td2, a, grid, s);
  else if (bn == 256) dispatch<256>(a_mn, b_mn, (int)epi, ta, tb, td, td2, a, grid, s);
  else dispatch<128>(a_mn, b_mn, (int)epi, ta, tb, td, td2, a, grid, s);
}

void gemm_bf16(torch::Tensor A, bool a_mn, torch::Tensor B, bool b_mn, int64_t M, int64_t N, int64_t K,
               torch::Tensor D, int64_t epi, double alpha, double beta, c10::optional<torch::Tensor> R,
               c10::optional<torch::Tensor> D2, double tau, int64_t split_k, int64_t bn, torch::Tensor err,
               c10::optional<torch::Tensor> alpha_t, double rcoef) {
  TORCH_CHECK(epi != EPI_ROPE && epi != EPI_CE, "the RoPE / CE epilogues are reached through gemm_rope / gemm_ce");
  gemm_bf16_impl(A, a_mn, B, b_mn, M, N, K, D, epi, alpha, beta, R, D2, tau, split_k, bn, err, alpha_t, rcoef,
                 RopeEpi{});
}

// D[M, N] = A[M, K] B[N, K]^T (bf16) with RoPE + per-head RMSNorm applied to the leading
// rope_cols columns (heads of 128; position = row % T; cos / sin [>= T][64] bf16) and the
// per-(row, head) reciprocal RMS written to rstd [M][rope_cols / 128] -- the q / k part of
// a fused QKV projection, the v columns stored as they are.
void gemm_rope(torch::Tensor A, torch::Tensor B, torch::Tensor D, torch::Tensor cos, torch::Tensor sin, int64_t T,
               int64_t rope_cols, c10::optional<torch::Tensor> rstd, torch::Tensor err) {
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && D.dim() == 2, "2-D operands");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && D.size(0) >= M && D.size(1) >= N, "shapes");
  TORCH_CHECK(rope_cols > 0 && rope_cols % 128 == 0 && rope_cols <= N, "rope_cols must be a multiple of 128 <= N");
  TORCH_CHECK(T > 0 && M % T == 0, "rows must be whole sequences of length T");
  for (const torch::Tensor* t : {&cos, &sin}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->dim() == 2 && t->size(1) == 64 &&
                    t->stride(1) == 1 && t->stride(0) == 64 && t->size(0) >= T,
                "cos / sin must be contiguous bf16 [>= T, 64]");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "cos / sin must be 16-byte aligned");
  }
  RopeEpi r;
  r.cos = reinterpret_cast<const __nv_bfloat16*>(cos.data_ptr());
  r.sin = reinterpret_cast<const __nv_bfloat16*>(sin.data_ptr());
  r.T = (int)T; r.cols = (int)rope_cols; r.heads = (int)(rope_cols / 128);
  if (rstd.has_value()) {
    TORCH_CHECK(rstd->is_cuda() && rstd->scalar_type() == at::kFloat && rstd->is_contiguous() &&
                    rstd->numel() >= M * r.heads,
                "rstd fp32 [M * heads]");
    r.rstd = rstd->data_ptr<float>();
  }
  gemm_bf16_impl(A, false, B, false, M, N, K, D, EPI_ROPE, 1.0, 0.0, c10::nullopt, c10::nullopt, 0.0, 1, 256, err,
                 c10::nullopt, 1.0, r);
}

// Row pass after the EPI_CE GEMM: one warp per row adds the row's partial sums, writes
// its loss w (S + log sum - y_c) and, with the gradient, rewrites the stored z as
// dz = w (exp(y - S) / sum - [j == c]) (1 - tanh(z / S)^2), 16-byte vectors.
__global__ void ce_finish_kernel(const __nv_bfloat16* __restrict__ zin, __nv_bfloat16* __restrict__ zout, long long ldz,
                                 int M, int N, int V, float S, const float* __restrict__ part, int parts,
                                 const float* __restrict__ yc, const void* __restrict__ tgt, int tgt_i64, int T,
                                 long long tgt_ld, const float* __restrict__ roww, float* __restrict__ loss,
                                 int write_dz) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const float invS = 1.f / S;
  float tot = 0.f;
  for (int k = lane; k < parts; k += 32) tot += part[(long long)row * parts + k];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  const long long ti = (long long)(row / T) * tgt_ld + row % T;
  const long long cls = tgt_i64 ? reinterpret_cast<const long long*>(tgt)[ti] : (long long)reinterpret_cast<const int*>(tgt)[ti];
  const bool valid = cls >= 0 && cls < V;
  const float wgt = valid ? (roww ? roww[row] : 1.f) : 0.f;
  if (lane == 0) loss[row] = valid ? wgt * (S + logf(tot) - yc[row]) : 0.f;
  if (!write_dz) return;
  const float inv_tot = 1.f / tot;
  const __nv_bfloat16* zr = zin + (long long)row * ldz;
  __nv_bfloat16* zw = zout + (long long)row * ldz;
  for (int j0 = lane * 8; j0 < N; j0 += 256) {
    uint4 u = *reinterpret_cast<const uint4*>(zr + j0);
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float2 z = __bfloat1622float2(h[q]);
      const float zz[2] = {z.x, z.y};
      float o[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = j0 + 2 * q + e;
        if (j < V && wgt != 0.f) {
          const float th = tanhf(zz[e] * invS);
          const float p = __expf(S * th - S) * inv_tot;
          o[e] = wgt * (p - (j == cls ? 1.f : 0.f)) * (1.f - th * th);
        } else {
          o[e] = 0.f;
        }
      }
      h[q] = __floats2bfloat162_rn(o[0], o[1]);
    }
    *reinterpret_cast<uint4*>(zw + j0) = u;
  }
}

// lm_head GEMM with the softcapped cross-entropy in the epilogue (EPI_CE).
//   A = x [M, K] bf16, B = W [N, K] bf16 (N = padded vocab, a multiple of 256, >= V);
//   tgt [B, T] int64 / int32 (row m = b * T + t; < 0 or >= V ignored); roww fp32 [M] or none;
//   part fp32 [M * 2 * ceil(N / 256)], yc fp32 [M] (scratch); loss fp32 [M] <-
//   w * (S + log sum_j exp(y_j - S) - y_c).
//   With write_dz, D [M, N] bf16 receives dz = w (softmax(y) - onehot)(1 - tanh^2) (scale 1;
//   the mean's 1 / denominator goes into the backward GEMMs' alpha); without, D is not
//   touched and may be any bf16 tensor.
void gemm_ce(torch::Tensor A, torch::Tensor B, torch::Tensor D, torch::Tensor tgt, int64_t T,
             c10::optional<torch::Tensor> roww, int64_t V, double S, torch::Tensor part, torch::Tensor yc,
             torch::Tensor loss, bool write_dz, torch::Tensor err) {
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && D.dim() == 2, "2-D operands");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K && N % 256 == 0 && V > 0 && V <= N, "N: padded vocab (multiple of 256) >= V");
  TORCH_CHECK(tgt.is_cuda() && (tgt.scalar_type() == at::kLong || tgt.scalar_type() == at::kInt) && tgt.dim() == 2 &&
                  tgt.stride(1) == 1 && T == tgt.size(1) && tgt.numel() == M,
              "targets [B, T] int64 / int32 with unit inner stride");
  const int64_t tiles_n = N / 256;
  TORCH_CHECK(part.scalar_type() == at::kFloat && part.numel() >= M * 2 * tiles_n, "part fp32 [M * 2 * tiles_n]");
  TORCH_CHECK(yc.scalar_type() == at::kFloat && yc.numel() >= M, "yc fp32 [M]");
  TORCH_CHECK(loss.scalar_type() == at::kFloat && loss.numel() >= M && loss.is_contiguous(), "loss fp32 [M]");
  if (write_dz) TORCH_CHECK(D.size(0) >= M && D.size(1) >= N, "D [M, N]");
  CeEpi c;
  c.tgt = tgt.data_ptr(); c.tgt_i64 = tgt.scalar_type() == at::kLong; c.T = (int)T; c.tgt_ld = tgt.stride(0);
  if (roww.has_value()) {
    TORCH_CHECK(roww->scalar_type() == at::kFloat && roww->numel() >= M && roww->is_contiguous(), "row weights fp32 [M]");
    c.roww = roww->data_ptr<float>();
  }
  c.V = (int)V; c.S = (float)S; c.part = part.data_ptr<float>(); c.yc = yc.data_ptr<float>();
  c.loss = loss.data_ptr<float>(); c.write_dz = write_dz ? 1 : 0;
  gemm_bf16_impl(A, false, B, false, M, N, K, D, EPI_CE, 1.0, 0.0, c10::nullopt, c10::nullopt, 0.0, 1, 256, err,
                 c10::nullopt, 1.0, RopeEpi{}, c);
  auto* z = reinterpret_cast<__nv_bfloat16*>(D.data_ptr());
  ce_finish_kernel<<<(unsigned)((M + 7) / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      z, z, D.stride(0), (int)M, (int)N, (int)V, (float)S, c.part, (int)(2 * tiles_n), c.yc, c.tgt, c.tgt_i64, c.T,
      c.tgt_ld, c.roww, c.loss, c.write_dz);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Few-row GEMM (decode): out[M, N] bf16 = x[M, K] W[N, K]^T (+ R | relu^2), K split over the
// SMs, partial sums added (vector atomics) into the zero-initialised fp32 workspace ws
// [M, N]; the last split of each region finishes it and re-zeroes ws / cnt (int32, >=
// tiles * 8 words, zero-initialised once).
void gemm_splitk_fin(torch::Tensor A, torch::Tensor B, torch::Tensor ws, torch::Tensor cnt, torch::Tensor out,
                     c10::optional<torch::Tensor> R, bool relu2, double tau, int64_t split, torch::Tensor err) {
  TORCH_CHECK(A.is_cuda() && A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1, "2-D operands");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "bf16 inputs");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "K mismatch");
  TORCH_CHECK(ws.scalar_type() == at::kFloat && ws.is_contiguous() && ws.size(0) >= M && ws.size(1) == N, "ws fp32 [M, N]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.size(0) >= M && out.size(1) >= N, "out bf16 [M, N]");
  TORCH_CHECK((out.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0 &&
                  (ws.stride(0) * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(ws.data_ptr()) & 15) == 0,
              "16-byte aligned rows");
  if (R.has_value())
    TORCH_CHECK((R->stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(R->data_ptr()) & 15) == 0,
                "residual rows must be 16-byte aligned");
  const int BM = 128, BK = 64, bn = 128;
  c10::cuda::CUDAGuard guard(A.device());
  CUtensorMap ta = make_tmap_bf16(A.data_ptr(), K, M, A.stride(0), 64, BM, 1, 0);
  CUtensorMap tb = make_tmap_bf16(B.data_ptr(), K, N, B.stride(0), 64, bn, 1, 0);
  GemmArgs a{};
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  a.tiles_m = (int)((M + BM - 1) / BM);
  a.tiles_n = (int)((N + bn - 1) / bn);
  a.kb_total = (int)((K + BK - 1) / BK);
  int sk = (int)std::max<int64_t>(1, std::min<int64_t>(split, a.kb_total));
  a.kb_per_split = (a.kb_total + sk - 1) / sk;
  sk = (a.kb_total + a.kb_per_split - 1) / a.kb_per_split;
  TORCH_CHECK(sk > 1, "split-K finish needs at least two splits");
  a.split_k = sk;
  a.batch = 1;
  a.num_tiles = a.tiles_m * a.tiles_n * sk;
  TORCH_CHECK(cnt.scalar_type() == at::kInt && cnt.numel() >= (int64_t)a.tiles_m * a.tiles_n * 8, "cnt int32 [tiles * 8]");
  a.alpha = 1.f; a.beta = 1.f; a.tau = (float)tau; a.rcoef = 1.f;
  a.alpha_ptr = nullptr;
  a.D = ws.data_ptr(); a.ldd = ws.stride(0); a.d_bstride = 0;
  a.D2 = nullptr; a.ldd2 = 0; a.d2_bstride = 0; a.R = nullptr; a.ldr = 0; a.r_bstride = 0;
  if (R.has_value()) {
    TORCH_CHECK(R->scalar_type() == at::kBFloat16 && R->stride(-1) == 1, "R must be bf16 row-major");
    a.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()); a.ldr = R->stride(0);
  }
  a.err = err.data_ptr<int>();
  a.tma_store = 0;
  a.fin_out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr()); a.ld_fin = out.stride(0);
  a.fin_cnt = cnt.data_ptr<int>();
  a.fin_relu2 = relu2 ? 1 : 0;
  const int grid = std::min(a.num_tiles, num_sms(A.get_device()));
  dispatch<128>(false, false, EPI_F32, ta, tb, ta, ta, a, grid, at::cuda::getCurrentCUDAStream());
}

// Tensor-parallel GEMMs with the collective fused in (MODE_AG / MODE_RS), A K-major.
//   AG: A = this rank's [M, K] gather buffer (rows [rank * Mr, (rank+1) * Mr) already
//       written); ag_src / ag_ready = every rank's gather-buffer base / ready pad;
//       claim [(world-1) * Mr / 128] and done [M / 128] are local uint32 words.
//       D [M, N] (and D2 / R as in the plain epilogues).
//   RS: D [Mr, N] bf16 = sum over ranks of (A B^T)[rank rows] (+ rcoef R), R [Mr, N];
//       rs_recv / rs_flag = every rank's receive buffer ([world][Mr][N] bf16) / flag
//       words ([world][Mr / 128 * tiles_n][8]: lane quarter x column half).
// sched: local uint32[2], zero before the first launch (the kernel leaves it zeroed).
// Every flag word holds the epoch of the last call that wrote it; epochs increase by
// one per call on every rank in the same order, starting above the words' initial 0.
void gemm_tp(int64_t mode, torch::Tensor A, torch::Tensor B, bool b_mn, int64_t M, int64_t N, int64_t K,
             torch::Tensor D, int64_t epi, c10::optional<torch::Tensor> R, c10::optional<torch::Tensor> D2,
             double tau, double rcoef, int64_t rank, int64_t world, int64_t rows_per_rank, int64_t epoch,
             std::vector<int64_t> ag_src, std::vector<int64_t> ag_ready, c10::optional<torch::Tensor> claim,
             c10::optional<torch::Tensor> done, std::vector<int64_t> rs_recv, std::vector<int64_t> rs_flag,
             torch::Tensor sched, int64_t bn, torch::Tensor err) {
  TORCH_CHECK(mode == MODE_AG || mode == MODE_RS, "mode must be AG (1) or RS (2)");
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && D.is_cuda() && A.dim() == 2 && B.dim() == 2 && D.dim() == 2, "2-D CUDA operands");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16 && D.scalar_type() == at::kBFloat16,
              "bf16 operands");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && D.stride(1) == 1, "inner dimension must be contiguous");
  TORCH_CHECK(world >= 1 && world <= kTpMaxRanks && rank >= 0 && rank < world, "rank / world");
  TORCH_CHECK(rows_per_rank % 128 == 0 && M == world * rows_per_rank, "M must be world x rows_per_rank, rows % 128 == 0");
  TORCH_CHECK(K % 8 == 0 && N > 0, "K must be a multiple of 8");
  TORCH_CHECK(A.size(0) >= M && A.size(1) >= K, "A shape");
  TORCH_CHECK(!b_mn ? (B.size(0) >= N && B.size(1) >= K) : (B.size(0) >= K && B.size(1) >= N), "B shape");
  TORCH_CHECK(sched.scalar_type() == at::kInt && sched.is_cuda() && sched.numel() >= 2, "sched int32[2]");
  TORCH_CHECK(bn == 128 || bn == 256, "bn must be 128 or 256");
  c10::cuda::CUDAGuard guard(A.device());
  const int BM = 128, BK = 64;
  CUtensorMap ta = make_tmap_bf16(A.data_ptr(), K, M, A.stride(0), 64, BM, 1, 0);
  CUtensorMap tb = !b_mn ? make_tmap_bf16(B.data_ptr(), K, N, B.stride(0), 64, (uint32_t)bn, 1, 0)
                         : make_tmap_bf16(B.data_ptr(), N, K, B.stride(0), 64, 64, 1, 0);
  GemmArgs a{};
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  a.tiles_m = (int)(M / BM);
  a.tiles_n = (int)((N + bn - 1) / bn);
  a.kb_total = (int)((K + BK - 1) / BK);
  a.kb_per_split = a.kb_total;
  a.split_k = 1;
  a.batch = 1;
  a.num_tiles = a.tiles_m * a.tiles_n;
  a.alpha = 1.f; a.beta = 0.f; a.tau = (float)tau; a.rcoef = (float)rcoef;
  a.alpha_ptr = nullptr;
  a.D = D.data_ptr(); a.ldd = D.stride(0); a.d_bstride = 0;
  a.D2 = nullptr; a.ldd2 = 0; a.d2_bstride = 0; a.R = nullptr; a.ldr = 0; a.r_bstride = 0;
  if (epi == EPI_RELU2) {
    TORCH_CHECK(D2.has_value() && D2->scalar_type() == at::kBFloat16 && D2->stride(-1) == 1, "RELU2 needs D2");
    a.D2 = D2->data_ptr(); a.ldd2 = D2->stride(0);
  }
  if (R.has_value()) {
    TORCH_CHECK(R->scalar_type() == at::kBFloat16 && R->stride(-1) == 1, "R must be bf16 row-major");
    a.R = reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()); a.ldr = R->stride(0);
  }
  TORCH_CHECK(epi != EPI_RELU2_BWD || a.R != nullptr, "RELU2_BWD needs R = pre-activation");
  a.err = err.data_ptr<int>();
  TpArgs& tp = a.tp;
  tp.rank = (int)rank; tp.world = (int)world; tp.rows_per_rank = (int)rows_per_rank; tp.epoch = (uint32_t)epoch;
  tp.sched = reinterpret_cast<uint32_t*>(sched.data_ptr<int>());
  if (mode == MODE_AG) {
    TORCH_CHECK((int64_t)ag_src.size() == world && (int64_t)ag_ready.size() == world, "one gather buffer / pad per rank");
    TORCH_CHECK(claim.has_value() && done.has_value() && claim->numel() >= (world - 1) * rows_per_rank / 128 &&
                    done->numel() >= M / 128, "claim / done words");
    TORCH_CHECK(D.size(0) >= M && D.size(1) >= N, "D shape");
    TORCH_CHECK((A.stride(0) * 2) % 16 == 0, "gather rows must be 16-byte aligned");
    for (int r = 0; r < world; ++r) {
      TORCH_CHECK((ag_src[r] & 15) == 0, "gather buffers must be 16-byte aligned");
      tp.ag_src[r] = reinterpret_cast<const uint8_t*>(ag_src[r]);
      tp.ag_ready[r] = reinterpret_cast<uint32_t*>(ag_ready[r]);
    }
    TORCH_CHECK(ag_src[rank] == reinterpret_cast<int64_t>(A.data_ptr()), "A must be this rank's gather buffer");
    tp.ag_dst = reinterpret_cast<uint8_t*>(A.data_ptr());
    tp.ag_ld_bytes = A.stride(0) * 2;
    tp.ag_row_bytes = (int)(K * 2);
    tp.ag_claim = reinterpret_cast<uint32_t*>(claim->data_ptr<int>());
    tp.ag_done = reinterpret_cast<uint32_t*>(done->data_ptr<int>());
  } else {
    TORCH_CHECK(epi == EPI_BF16, "reduce-scatter epilogue is bf16 (+ residual)");
    TORCH_CHECK((int64_t)rs_recv.size() == world && (int64_t)rs_flag.size() == world, "one receive buffer / flag array per rank");
    TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8 (16-byte receive rows)");
    TORCH_CHECK(D.size(0) >= rows_per_rank && D.size(1) >= N, "D shape");
    if (a.R) TORCH_CHECK(R->size(0) >= rows_per_rank && R->size(1) >= N, "R shape");
    for (int r = 0; r < world; ++r) {
      TORCH_CHECK((rs_recv[r] & 15) == 0 && (rs_flag[r] & 3) == 0, "receive buffers 16-byte, flags 4-byte aligned");
      tp.rs_recv[r] = reinterpret_cast<__nv_bfloat16*>(rs_recv[r]);
      tp.rs_flag[r] = reinterpret_cast<uint32_t*>(rs_flag[r]);
    }
  }
  CUtensorMap td = ta, td2 = ta;
  a.tma_store = 0;
  if (mode == MODE_AG && tma_store_ok(epi, N, a.D, a.ldd, 0, epi == EPI_RELU2 ? a.D2 : nullptr, a.ldd2, 0)) {
    a.tma_store = 1;
    td = make_tmap_bf16(a.D, N, M, a.ldd, 64, 32, 1, 0);
    if (epi == EPI_RELU2) td2 = make_tmap_bf16(a.D2, N, M, a.ldd2, 64, 32, 1, 0);
  }
  const int grid = std::min(a.num_tiles, num_sms(A.get_device()));
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (bn == 256) dispatch_tp<256>((int)mode, b_mn, (int)epi, ta, tb, td, td2, a, grid, s);
  else dispatch_tp<128>((int)mode, b_mn, (int)epi, ta, tb, td, td2, a, grid, s);
}

}  // namespace tfb
