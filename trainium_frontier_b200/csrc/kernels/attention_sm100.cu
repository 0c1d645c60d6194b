// Causal flash attention, forward and backward, on the 5th-generation tensor cores.
//
// Layout: q, k, v are row views [B*T, *] with head h at columns [h*D, h*D + D) (the
// projection buffers are read in place -- no transposes).  T % 128 == 0, D in {64, 128}.
//
// Forward: one CTA per (batch*head, 128-query tile), heaviest tiles first.
//   warp 0   TMA: Q once, K/V tiles double-buffered
//   warp 1   MMA: S_j = Q K_j^T -> TMEM (double-buffered), O += P_j V_j -> TMEM
//   warps 2-5 softmax: one query row per thread (= TMEM lane).  Row max / exp2 / sum in
//            registers, P written to shared memory in the 128B-swizzled K-major layout the
//            P*V MMA reads; O is rescaled in TMEM (ld/st) only when a warp's max moved.
//            Epilogue: O / l -> bf16, LSE (natural log) for the backward.
// Backward: one CTA per (batch*head, 128-key tile), in the transposed frame so every
//   per-row operation is again one TMEM lane per thread:
//     S^T = K Q_i^T, dP^T = V dO_i^T                      (TMEM)
//     P^T = exp(S^T * scale - LSE_i), dS^T = P^T (dP^T - Dvec_i)   (registers -> smem)
//     dV += P^T dO_i, dK += dS^T Q_i                       (TMEM accumulators)
//     dQ_i = dS K  -> fp32 vector atomics into a dQ accumulator
// Faster forms for head_dim 128 (below): a two-query-tile forward that ping-pongs two
// softmax warpgroups on the tensor core, and a pipelined backward (double-buffered Q / dO,
// dQ drained by dedicated warps).  TFB_FA_FWD_ONE_TILE / TFB_FA_BWD_SERIAL select the
// simple forms above (kept as the reference the fast forms are tested against).
// Every wait is bounded (see sm100_common.cuh); every TMA load is a plain per-CTA load.
// Reference counterparts: the SDPA call of CausalSelfAttention (train.py:2564-2567) and the
// research NKI kernels research/scratch/nki_attn_fwd.py:41-132 and nki_attn_bwd.py:1-367.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

CUtensorMap make_tmap_bf16(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                           uint32_t box_inner, uint32_t box_outer, uint64_t batch, uint64_t batch_stride_elems);
CUtensorMap make_tmap_f32(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                          uint32_t box_inner, uint32_t box_outer);

struct FaArgs {
  int B, T, H, n_tiles, causal;
  float scale, scale_log2;
  __nv_bfloat16* O;
  long long ldo;
  float* lse;
  const float* dvec;
  float* dq_acc;
  long long lddq;
  __nv_bfloat16* dK;
  long long lddk;
  __nv_bfloat16* dV;
  long long lddv;
  int* err;
  long long* trace;  // optional phase timeline (clock64) of CTA 0, see fa_trace_set
};

// Phase timeline of CTA 0 (off unless a buffer is installed): role r, step i, event e at
// trace[(r * 64 + i) * 8 + e], i < 64.  Roles: 0 MMA issuer, 1 softmax warp (first of
// its group), 2 dQ drain / second softmax group, 3 producer.
__device__ __forceinline__ void fa_stamp(long long* tr, int role, int i, int e) {
  if (tr != nullptr && blockIdx.x == 0 && i < 64) tr[(role * 64 + i) * 8 + e] = clock64();
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr uint32_t kPanel = 128u * 128u;  // one 64-column panel of 128 rows (bytes)

template <int D>
struct FaCfg {
  static constexpr int PANELS = D / 64;
  static constexpr uint32_t TILE = 128u * D * 2u;     // 128 rows x D bf16
  static constexpr uint32_t PTILE = 128u * 128u * 2u;  // 128 x 128 bf16
  static constexpr size_t FWD_SMEM = 1024 + TILE * 5 + PTILE + 16 * 8 + 16;
  static constexpr size_t BWD_SMEM = 1024 + TILE * 4 + PTILE * 2 + 2 * 128 * 4 + 20 * 8 + 16;
};

// Grid order of the two-tile forward and pipelined backward: work items (head, tile) are
// taken in groups of G heads with G * tiles ~ 128 CTAs, heaviest tiles first inside a
// group and heads fastest.  The CTAs resident at any time then cover a few heads whole,
// so each K / V (forward) or Q / dO (backward) tile is read from HBM once and served to
// that head's other CTAs from L2, instead of every CTA streaming its own head.
__device__ __forceinline__ void grouped_item(int idx, int BH, int tiles, bool heavy_high, int& bh, int& tile) {
  const int G = max(1, 128 / tiles);
  const int group = idx / (G * tiles);
  const int g0 = group * G;
  const int gsz = min(G, BH - g0);
  const int r = idx - group * G * tiles;
  const int t = r / gsz;
  bh = g0 + r % gsz;
  tile = heavy_high ? tiles - 1 - t : t;
}

// K-major operand tile with K = 128 elements (two 64-element panels): k-step kk of 16.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int kk) {
  return umma_desc_sw128(base + (uint32_t)(kk >> 2) * kPanel + (uint32_t)(kk & 3) * 32u, 16, 1024);
}
// MN-major operand tile (MN in 64-element panels, K along the 128 rows): k-step kk of 16.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int kk) {
  return umma_desc_sw128(base + (uint32_t)kk * 2048u, kPanel, 1024);
}

// Write 128 fp32 values (one row) as bf16 into a 128-row x 128-col swizzled tile.
__device__ __forceinline__ void store_row_bf16_sw128(uint8_t* tile, int row, const float* v) {
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    u.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    u.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    u.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(tile + (c >> 3) * kPanel + sw128_chunk_offset(row, c & 7)) = u;
  }
}

__device__ __forceinline__ void store_row_bf16_global(__nv_bfloat16* dst, const float* v, int n) {
  for (int c = 0; c < n / 8; ++c) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    u.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    u.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    u.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    reinterpret_cast<uint4*>(dst)[c] = u;
  }
}

// ================================================================================ forward
template <int D>
__global__ void __launch_bounds__(192, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const FaArgs a) {
  using Cfg = FaCfg<D>;
  constexpr uint32_t TILE = Cfg::TILE;
  constexpr uint32_t IDESC_S = umma_idesc_bf16(128, 128, false, false);
  constexpr uint32_t IDESC_O = umma_idesc_bf16(128, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + TILE;
  uint8_t* sV = sK + 2 * TILE;
  uint8_t* sP = sV + 2 * TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + Cfg::PTILE);
  uint64_t* bar_q = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = a.B * a.H;
  const int qt = a.n_tiles - 1 - (int)(blockIdx.x / BH);
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / a.H, h = bh % a.H;
  const int row0 = b * a.T + qt * 128;
  const int n_kv = a.causal ? qt + 1 : a.n_tiles;

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      uint32_t out_valid = 0, out_parity = 0;
      mbar_arrive_expect_tx(bar_q, TILE);
#pragma unroll
      for (int p = 0; p < Cfg::PANELS; ++p) tma_load_3d(sQ + p * kPanel, &tmQ, bar_q, h * D + p * 64, row0, 0);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[s], ((j - 2) >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[s], 2 * TILE);
        out_valid |= 1u << s;
        out_parity = (out_parity & ~(1u << s)) | ((uint32_t)((j >> 1) & 1) << s);
        const int krow = b * a.T + j * 128;
#pragma unroll
        for (int p = 0; p < Cfg::PANELS; ++p) {
          tma_load_3d(sK + s * TILE + p * kPanel, &tmK, &kv_full[s], h * D + p * 64, krow, 0);
          tma_load_3d(sV + s * TILE + p * kPanel, &tmV, &kv_full[s], h * D + p * 64, krow, 0);
        }
      }
      if (!ok) {
        for (int s = 0; s < 2; ++s) {
          if (!((out_valid >> s) & 1u)) continue;
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&kv_full[s], (out_parity >> s) & 1u))
            if (globaltimer_ns() - t0 > 100000000ull) break;
        }
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_q, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(bar_q, 0, abort_flag, a.err, ERR_TIMEOUT_MMA);
      const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait(p_full, jj & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (jj & 1) * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tO, desc_kmajor(p_addr, kk), desc_mnmajor(v_addr, kk), IDESC_O, (jj > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[jj & 1]);
        umma_commit(pv_done);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_full[s], (j >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        if (j >= 2 && !mbar_wait(&s_free[s], ((j - 2) >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_bf16(tS[s], desc_kmajor(q_addr, kk), desc_kmajor(k_addr, kk), IDESC_S, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[s]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_pv(n_kv - 1);
      if (!ok) {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      if (!mbar_wait_warp(&s_full[s], (j >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      float x[128];
      {
        uint32_t* xr = reinterpret_cast<uint32_t*>(x);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          __syncwarp();
          tmem_ld_32x32b_x32(tS[s] + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(xr + 32 * c));
        }
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(&s_free[s]);
      const bool diag = a.causal && (j == qt);
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        float t = x[i] * a.scale_log2;
        if (diag && i > r) t = -INFINITY;
        x[i] = t;
        mx = fmaxf(mx, t);
      }
      const float m_new = fmaxf(m, mx);
      const float alpha = exp2f(m - m_new);
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        const float pv = exp2f(x[i] - m_new);
        x[i] = pv;
        sum += pv;
      }
      l = l * alpha + sum;
      m = m_new;
      if (j >= 1) {
        if (!mbar_wait_warp(pv_done, (j - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha < 1.f)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            __syncwarp();
            tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st_32x32b_x32(tO + lane_off + c * 32, o);
          }
          tmem_st_wait();
        }
      }
      store_row_bf16_sw128(sP, r, x);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait_warp(pv_done, (n_kv - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      __nv_bfloat16* dst = a.O + (long long)(row0 + r) * a.ldo + h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
        tmem_ld_wait();
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(o[i]) * inv_l;
        store_row_bf16_global(dst + c * 32, f, 32);
      }
      a.lse[(long long)bh * a.T + qt * 128 + r] = (m + log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================================ forward, two Q tiles
// One CTA per (batch*head, pair of 128-query tiles), heaviest pairs first.  The two tiles
// share every K/V tile load and ping-pong on the tensor core: while softmax warpgroup 0
// turns S0 = Q0 K_j^T into P0, the MMA warp runs S1 / P1 V for tile 1, and vice versa.
//   warp 0      TMA: Q0 + Q1 once, then K_0, V_0, K_1, V_1, ... through a 4-slot ring, so
//               each K / V load has more than a full step of lead before its MMA
//   warp 1      MMA: S0(j+1), P0 V(j), S1(j+1), P1 V(j) per step j
//   warps 2-5   softmax of tile 0 (one query row per thread = TMEM lane)
//   warps 6-9   softmax of tile 1
// The two groups write P into ONE shared-memory tile in turn (P0(j), P1(j), P0(j+1), ...):
// each waits for the P V MMA of the other tile's previous turn, which the ping-pong order
// has already issued, and the 32 KB saved go to the K / V ring.
// TMEM: S0 | S1 | O0 | O1 (4 x 128 columns).  The row max used as the exponent reference
// only moves when it grows by more than 8 (log2 units), so O is rarely rescaled; p values
// stay below 2^8.  Softmax math runs on packed fp32 pairs (fma / add .f32x2) with a
// three-input max; a quarter of the exponentials is computed on the FMA pipe
// (exp2_poly) so the MUFU unit, whose 16 results per clock per SM match the tensor core's
// 16 score elements per clock at head_dim 128, is not the limit.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^v on the FMA pipe for v <= 8 (0 below -126): v = n + f with n the nearest integer
// (added and subtracted 1.5 * 2^23, whose low mantissa bits then hold n) and f in
// [-1/2, 1/2]; 2^f from a degree-3 polynomial fitted here for relative error on that
// interval (max relative error 7.5e-5, far below the bf16 rounding of P); 2^n added
// into the exponent field as n << 23, which is the magic sum's bits shifted by 23.
// Clamping v at -126 keeps that exponent field from underflowing.
__device__ __forceinline__ float2 exp2_poly2(float2 v) {
  const float2 vc = make_float2(fmaxf(v.x, -126.f), fmaxf(v.y, -126.f));
  const float2 t = __fadd2_rn(vc, make_float2(12582912.f, 12582912.f));
  const float2 n = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __fadd2_rn(vc, make_float2(-n.x, -n.y));
  float2 p = __ffma2_rn(make_float2(0.055170949548482895f, 0.055170949548482895f), f,
                        make_float2(0.2426096349954605f, 0.2426096349954605f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999281764030457f, 0.9999281764030457f));
  const float rx = __int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23));
  const float ry = __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23));
  return make_float2(v.x < -126.f ? 0.f : rx, v.y < -126.f ? 0.f : ry);
}

constexpr int kFwd2Slots = 5;  // K / V ring depth
constexpr size_t kFwd2Smem = 1024 + 2 * 32768 + kFwd2Slots * 32768 + 24 * 8 + 16;

// Two 128-query tiles per CTA, K/V streamed through a 5-slot TMA ring; TMEM holds S_t and
// O_t for both tiles (4 x 128 columns).  The softmax of tile t writes P_t (bf16) back into
// the first 64 columns of S_t and the P V MMA reads it from TMEM as its A operand, so P
// never goes through shared memory.  Since S_t(j+1) would overwrite P_t(j), the MMA warp
// issues S_t(j+1) right after P_t(j) V_j (tcgen05 MMAs of one thread run in issue order);
// the two tiles alternate, so the tensor pipe runs one tile's P V and next S while the
// other tile's softmax runs.  The commit that signals S_t(j) also covers P_t(j-1) V_{j-1},
// so the softmax may rescale O_t as soon as it sees S_t(j).
__global__ void __launch_bounds__(320, 1)
    fa_fwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const FaArgs a) {
  constexpr int D = 128;
  constexpr uint32_t TILE = 128u * D * 2u;
  constexpr uint32_t IDESC_S = umma_idesc_bf16(128, 128, false, false);
  constexpr uint32_t IDESC_O = umma_idesc_bf16(128, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int NS = kFwd2Slots;
  uint8_t* sQ = smem;                 // [2] tiles
  uint8_t* sKV = sQ + 2 * TILE;       // [NS] slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + NS * TILE);
  uint64_t* bar_q = bars + 0;
  uint64_t* kv_full = bars + 1;          // [NS]
  uint64_t* kv_empty = bars + 1 + NS;    // [NS]
  uint64_t* s_full = bars + 1 + 2 * NS;  // [2]
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_done = p_full + 2;         // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = a.B * a.H;
  const int n_pairs = a.n_tiles >> 1;
  int pc, bh;
  grouped_item((int)blockIdx.x, BH, n_pairs, true, bh, pc);
  const int b = bh / a.H, h = bh % a.H;
  const int qt0 = 2 * pc;
  const int row0 = b * a.T + qt0 * 128;
  const int n0 = a.causal ? qt0 + 1 : a.n_tiles;   // K/V tiles of tile 0
  const int n1 = a.causal ? qt0 + 2 : a.n_tiles;   // ... of tile 1 (>= n0)

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      uint32_t out_valid = 0, out_parity = 0;
      mbar_arrive_expect_tx(bar_q, 2 * TILE);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int p = 0; p < 2; ++p)
          tma_load_3d(sQ + t * TILE + p * kPanel, &tmQ, bar_q, h * D + p * 64, row0 + t * 128, 0);
      const int items = 2 * n1;
      for (int i = 0; i < items && ok; ++i) {
        const int slot = i % NS;
        if (i >= NS && !mbar_wait(&kv_empty[slot], ((i / NS) + 1) & 1, abort_flag, a.err, ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&kv_full[slot], TILE);
        out_valid |= 1u << slot;
        out_parity = (out_parity & ~(1u << slot)) | ((uint32_t)((i / NS) & 1) << slot);
        const int krow = b * a.T + (i >> 1) * 128;
        const CUtensorMap* map = (i & 1) ? &tmV : &tmK;
#pragma unroll
        for (int p = 0; p < 2; ++p) tma_load_3d(sKV + slot * TILE + p * kPanel, map, &kv_full[slot], h * D + p * 64, krow, 0);
      }
      if (!ok) {
        for (int s = 0; s < NS; ++s) {
          if (!((out_valid >> s) & 1u)) continue;
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&kv_full[s], (out_parity >> s) & 1u))
            if (globaltimer_ns() - t0 > 100000000ull) break;
        }
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(bar_q, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(bar_q, 0, abort_flag, a.err, ERR_TIMEOUT_MMA);
      const uint32_t q_addr[2] = {smem_u32(sQ), smem_u32(sQ + TILE)};
      auto kv_wait = [&](int item) -> bool {
        return mbar_wait(&kv_full[item % NS], (item / NS) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA);
      };
      auto issue_s = [&](int t, int j) -> bool {
        if (!kv_wait(2 * j)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + ((2 * j) % NS) * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_bf16(tmem + t * 128, desc_kmajor(q_addr[t], kk), desc_kmajor(k_addr, kk), IDESC_S, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[t]);
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        if (!kv_wait(2 * j + 1)) return false;
        if (!mbar_wait(&p_full[t], j & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sKV + ((2 * j + 1) % NS) * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // P_t(j): 16 keys = 8 packed columns per MMA
          umma_bf16_tmem_a(tmem + 256 + t * 128, tmem + t * 128 + kk * 8, desc_mnmajor(v_addr, kk), IDESC_O,
                           (j > 0 || kk > 0) ? 1u : 0u);
        return true;
      };
      if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
      if (ok) umma_commit(&kv_empty[0]);  // K_0 read by both tiles
      for (int j = 0; j < n1 && ok; ++j) {
        fa_stamp(a.trace, 0, j, 0);
        if (j < n0) {
          if (!issue_pv(0, j)) { ok = false; break; }
          fa_stamp(a.trace, 0, j, 1);
          if (j + 1 < n0) {
            if (!issue_s(0, j + 1)) { ok = false; break; }
          } else {
            umma_commit(&o_done[0]);
          }
          fa_stamp(a.trace, 0, j, 2);
        }
        if (!issue_pv(1, j)) { ok = false; break; }
        fa_stamp(a.trace, 0, j, 3);
        if (j + 1 < n1) {
          if (!issue_s(1, j + 1)) { ok = false; break; }
          umma_commit(&kv_empty[(2 * (j + 1)) % NS]);  // K_{j+1} read by both tiles
        } else {
          umma_commit(&o_done[1]);
        }
        fa_stamp(a.trace, 0, j, 4);
        umma_commit(&kv_empty[(2 * j + 1) % NS]);      // V_j done
      }
      if (!ok) {
        *abort_flag = 1;
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax (tile t)
    const int t = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t tS = tmem + t * 128, tO = tmem + 256 + t * 128;
    const int n_t = t == 0 ? n0 : n1;
    const int qt = qt0 + t;
    const float c = a.scale_log2;
    float m_run = -INFINITY, l = 0.f;
    bool ok = true;
    const bool stamp = (warp == 2 || warp == 6) && lane == 0;
    for (int j = 0; j < n_t; ++j) {
      if (stamp) fa_stamp(a.trace, 1 + t, j, 0);
      if (!mbar_wait_warp(&s_full[t], j & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (stamp) fa_stamp(a.trace, 1 + t, j, 1);
      tc_fence_after();
      float x[128];
      {
        uint32_t* xr = reinterpret_cast<uint32_t*>(x);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          __syncwarp();
          tmem_ld_32x32b_x32(tS + lane_off + cc * 32, *reinterpret_cast<uint32_t(*)[32]>(xr + 32 * cc));
        }
        tmem_ld_wait();
      }
      if (a.causal && j == qt) {  // diagonal tile: keys after this query row are masked
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > r) x[i] = -INFINITY;
      }
      // four independent max chains, two new elements per three-input max
      float mx4[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
      for (int i = 4; i < 128; i += 8)
#pragma unroll
        for (int k = 0; k < 4; ++k) mx4[k] = max3f(mx4[k], x[i + k], x[i + 4 + k]);
      const float mxs = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * c;
      float alpha = 1.f;
      const bool grow = mxs > m_run + 8.f;
      if (grow) {
        alpha = ex2_approx(m_run - mxs);
        m_run = mxs;
      }
      // p = 2^(x c - m): packed pairs; columns 96..127 of every row on the FMA pipe
      const float2 c2 = make_float2(c, c), nm2 = make_float2(-m_run, -m_run);
      float2 sm4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t pk[64];  // the row of P as packed bf16 pairs
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        const float2 v = __ffma2_rn(make_float2(x[i], x[i + 1]), c2, nm2);
        float2 p2;
        if (i >= 96) p2 = exp2_poly2(v);
        else p2 = make_float2(ex2_approx(v.x), ex2_approx(v.y));
        pk[i >> 1] = pack_bf16x2(p2.x, p2.y);
        sm4[(i >> 1) & 3] = __fadd2_rn(sm4[(i >> 1) & 3], p2);
      }
      const float2 s01 = __fadd2_rn(__fadd2_rn(sm4[0], sm4[1]), __fadd2_rn(sm4[2], sm4[3]));
      l = l * alpha + (s01.x + s01.y);
      if (stamp) fa_stamp(a.trace, 1 + t, j, 2);
      // O_t is stable: the commit that signalled S_t(j) covered P_t(j-1) V_{j-1}
      if (j >= 1 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          __syncwarp();
          tmem_ld_32x32b_x32(tO + lane_off + cc * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st_32x32b_x32(tO + lane_off + cc * 32, o);
        }
      }
      if (stamp) fa_stamp(a.trace, 1 + t, j, 3);
      // P_t(j) over the first 64 columns of S_t(j) (already in registers)
      __syncwarp();
      tmem_st_32x32b_x32(tS + lane_off, *reinterpret_cast<const uint32_t(*)[32]>(pk));
      tmem_st_32x32b_x32(tS + lane_off + 32, *reinterpret_cast<const uint32_t(*)[32]>(pk + 32));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      if (stamp) fa_stamp(a.trace, 1 + t, j, 4);
    }
    if (ok && mbar_wait_warp(&o_done[t], 0, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      const float inv_l = 1.f / l;
      __nv_bfloat16* dst = a.O + (long long)(row0 + t * 128 + r) * a.ldo + h * D;
#pragma unroll 1
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tO + lane_off + cc * 32, o);
        tmem_ld_wait();
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(o[i]) * inv_l;
        store_row_bf16_global(dst + cc * 32, f, 32);
      }
      a.lse[(long long)bh * a.T + qt * 128 + r] = (m_run + log2f(l)) * kLn2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================================ backward
template <int D>
__global__ void __launch_bounds__(192, 1)
    fa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO, const FaArgs a) {
  using Cfg = FaCfg<D>;
  constexpr uint32_t TILE = Cfg::TILE;
  constexpr uint32_t IDESC_SS = umma_idesc_bf16(128, 128, false, false);  // S^T, dP^T
  constexpr uint32_t IDESC_KV = umma_idesc_bf16(128, D, false, true);     // dV, dK
  constexpr uint32_t IDESC_Q = umma_idesc_bf16(128, D, true, true);       // dQ

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  uint8_t* sQ = sV + TILE;
  uint8_t* sDO = sQ + TILE;
  uint8_t* sP = sDO + TILE;
  uint8_t* sDS = sP + Cfg::PTILE;
  float* sLse = reinterpret_cast<float*>(sDS + Cfg::PTILE);
  float* sDv = sLse + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDv + 128);
  uint64_t* bar_kv = bars + 0;
  uint64_t* qdo_full = bars + 1;
  uint64_t* qdo_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* dp_full = bars + 4;
  uint64_t* p_full = bars + 5;
  uint64_t* ds_full = bars + 6;
  uint64_t* dq_full = bars + 7;
  uint64_t* dq_free = bars + 8;
  uint64_t* dp_free = bars + 9;
  uint64_t* kv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = a.B * a.H;
  const int kt = (int)(blockIdx.x / BH);  // small key tiles have the most work: first
  const int bh = (int)(blockIdx.x % BH);
  const int b = bh / a.H, h = bh % a.H;
  const int krow0 = b * a.T + kt * 128;
  const int i0 = a.causal ? kt : 0;
  const int n_it = a.n_tiles - i0;

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    mbar_init(qdo_full, 1);
    mbar_init(qdo_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_full, 128);
    mbar_init(ds_full, 128);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(dp_free, 128);
    mbar_init(kv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tA = tmem;        // S^T, then dQ
  const uint32_t tB = tmem + 128;  // dP^T
  const uint32_t tDV = tmem + 256;
  const uint32_t tDK = tmem + 256 + D;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      bool pending = false;
      uint32_t pend_par = 0;
      mbar_arrive_expect_tx(bar_kv, 2 * TILE);
#pragma unroll
      for (int p = 0; p < Cfg::PANELS; ++p) {
        tma_load_3d(sK + p * kPanel, &tmK, bar_kv, h * D + p * 64, krow0, 0);
        tma_load_3d(sV + p * kPanel, &tmV, bar_kv, h * D + p * 64, krow0, 0);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        if (it >= 1 && !mbar_wait(qdo_empty, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx(qdo_full, 2 * TILE + 2 * 512);
        pending = true;
        pend_par = it & 1;
        const int qrow = b * a.T + (i0 + it) * 128;
        bulk_load(sLse, a.lse + (long long)bh * a.T + (i0 + it) * 128, 512, qdo_full);
        bulk_load(sDv, a.dvec + (long long)bh * a.T + (i0 + it) * 128, 512, qdo_full);
#pragma unroll
        for (int p = 0; p < Cfg::PANELS; ++p) {
          tma_load_3d(sQ + p * kPanel, &tmQ, qdo_full, h * D + p * 64, qrow, 0);
          tma_load_3d(sDO + p * kPanel, &tmDO, qdo_full, h * D + p * 64, qrow, 0);
        }
      }
      if (!ok) {
        const unsigned long long t0 = globaltimer_ns();
        while (pending && !mbar_try_wait(qdo_full, pend_par))
          if (globaltimer_ns() - t0 > 100000000ull) break;
        while (!mbar_try_wait(bar_kv, 0))
          if (globaltimer_ns() - t0 > 200000000ull) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(bar_kv, 0, abort_flag, a.err, ERR_TIMEOUT_MMA);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
      const uint32_t p_addr = smem_u32(sP), ds_addr = smem_u32(sDS);
      for (int it = 0; it < n_it && ok; ++it) {
        if (!mbar_wait(qdo_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        if (it >= 1 && !mbar_wait(dq_free, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // S^T = K Q^T
          umma_bf16(tA, desc_kmajor(k_addr, kk), desc_kmajor(q_addr, kk), IDESC_SS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        if (it >= 1 && !mbar_wait(dp_free, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // dP^T = V dO^T
          umma_bf16(tB, desc_kmajor(v_addr, kk), desc_kmajor(do_addr, kk), IDESC_SS, kk > 0 ? 1u : 0u);
        umma_commit(dp_full);
        if (!mbar_wait(p_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO
          umma_bf16(tDV, desc_kmajor(p_addr, kk), desc_mnmajor(do_addr, kk), IDESC_KV, (it > 0 || kk > 0) ? 1u : 0u);
        if (!mbar_wait(ds_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dK += dS^T Q
          umma_bf16(tDK, desc_kmajor(ds_addr, kk), desc_mnmajor(q_addr, kk), IDESC_KV, (it > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dQ = dS K
          umma_bf16(tA, desc_mnmajor(ds_addr, kk), desc_mnmajor(k_addr, kk), IDESC_Q, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(qdo_empty);
      }
      if (ok) umma_commit(kv_done);
      else {
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int i = i0 + it;
      // LSE / Dvec of this query tile arrive with Q and dO (same barrier)
      if (!mbar_wait_warp(qdo_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (!mbar_wait_warp(s_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      const bool diag = a.causal && (i == kt);
      uint32_t pk[64];  // P^T row as packed bf16 pairs (kept for dS)
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t sv[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tA + lane_off + c4 * 32, sv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int c = c4 * 32 + e;
          float p0 = exp2f(__uint_as_float(sv[e]) * a.scale_log2 - sLse[c] * kLog2e);
          float p1 = exp2f(__uint_as_float(sv[e + 1]) * a.scale_log2 - sLse[c + 1] * kLog2e);
          if (diag && c < r) p0 = 0.f;  // query c precedes key r: no attention
          if (diag && c + 1 < r) p1 = 0.f;
          pk[c >> 1] = pack_bf16x2(p0, p1);
        }
      }
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 u = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4*>(sP + (c >> 3) * kPanel + sw128_chunk_offset(r, c & 7)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      if (!mbar_wait_warp(dp_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t dv[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tB + lane_off + c4 * 32, dv);
        tmem_ld_wait();
        uint32_t dsk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int c = c4 * 32 + e;
          const float2 pf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk[c >> 1]));
          dsk[e >> 1] = pack_bf16x2(pf.x * (__uint_as_float(dv[e]) - sDv[c]),
                                    pf.y * (__uint_as_float(dv[e + 1]) - sDv[c + 1]));
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = c4 * 4 + q;  // 16-byte chunk index within the 128-column row
          *reinterpret_cast<uint4*>(sDS + (c >> 3) * kPanel + sw128_chunk_offset(r, c & 7)) =
              make_uint4(dsk[4 * q], dsk[4 * q + 1], dsk[4 * q + 2], dsk[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(dp_free);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      if (!mbar_wait_warp(dq_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      float* dq = a.dq_acc + (long long)(b * a.T + i * 128 + r) * a.lddq + h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tA + lane_off + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 8; ++v)
          atomicAdd(reinterpret_cast<float4*>(dq + c * 32) + v,
                    make_float4(__uint_as_float(o[4 * v]) * a.scale, __uint_as_float(o[4 * v + 1]) * a.scale,
                                __uint_as_float(o[4 * v + 2]) * a.scale, __uint_as_float(o[4 * v + 3]) * a.scale));
      }
      tc_fence_before();
      mbar_arrive(dq_free);
    }
    if (ok && mbar_wait_warp(kv_done, 0, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      __nv_bfloat16* dv = a.dV + (long long)(krow0 + r) * a.lddv + h * D;
      __nv_bfloat16* dk = a.dK + (long long)(krow0 + r) * a.lddk + h * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        float f[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tDV + lane_off + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 32; ++v) f[v] = __uint_as_float(o[v]);
        store_row_bf16_global(dv + c * 32, f, 32);
        __syncwarp();
        tmem_ld_32x32b_x32(tDK + lane_off + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 32; ++v) f[v] = __uint_as_float(o[v]) * a.scale;
        store_row_bf16_global(dk + c * 32, f, 32);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================================ backward, pipelined
// D = 128.  One CTA per (batch*head, 128-key tile), transposed frame as above, but:
//   * Q_i / LSE_i / Dvec_i are double-buffered (tile i+1 loads during tile i); dO_i is
//     single-buffered and reloaded as soon as the dV MMA of tile i has read it;
//   * P^T and dS^T share one shared-memory tile (dS is written once the dV MMA has read P);
//   * TMEM: R0 = S^T, R1 = dP^T then dQ, dV, dK.  S^T(i+1) is issued right after dV(i),
//     before the wait for dS(i); dQ(i) lands in R1 once dP^T(i) has been read;
//   * four dedicated warps drain dQ: 32-column slices are staged (scaled, 128-byte swizzle)
//     in a double-buffered shared tile and added into the fp32 dQ accumulator by TMA bulk
//     reduce-adds, so no per-thread global atomics remain.
//   warp 0 TMA, warp 1 MMA, warps 2-9 softmax / dS / epilogue (two per TMEM lane quarter,
//   64 columns each), warps 10-13 dQ drain.
constexpr size_t kBwd2Need = 2 * 32768 + 2 * 32768 + 32768 + 32768 + 2 * 16384 + 4 * 512 + 32 * 8 + 32;
constexpr size_t kBwd2Smem = 232448;

__global__ void __launch_bounds__(448, 1)
    fa_bwd2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmDQ, const FaArgs a) {
  constexpr int D = 128;
  constexpr uint32_t TILE = 128u * D * 2u;
  constexpr uint32_t STG = 128u * 32u * 4u;  // one 32-column fp32 dQ slice
  constexpr uint32_t IDESC_SS = umma_idesc_bf16(128, 128, false, false);  // S^T, dP^T
  constexpr uint32_t IDESC_KV = umma_idesc_bf16(128, D, false, true);     // dV, dK
  constexpr uint32_t IDESC_Q = umma_idesc_bf16(128, D, true, true);       // dQ

  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad + kBwd2Need > kBwd2Smem) {  // dynamic shared memory base too poorly aligned
    if (threadIdx.x == 0) atomicOr(a.err, ERR_BAD_ARG);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE;
  uint8_t* sQ = sV + TILE;          // [2]
  uint8_t* sDO = sQ + 2 * TILE;     // [1]
  uint8_t* sPD = sDO + TILE;        // P^T, then dS^T
  uint8_t* sDQ = sPD + TILE;        // [2] dQ staging slices
  float* sLse = reinterpret_cast<float*>(sDQ + 2 * STG);  // [2][128]
  float* sDv = sLse + 256;                                // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDv + 256);
  uint64_t* bar_kv = bars + 0;
  uint64_t* q_full = bars + 1;     // [2]
  uint64_t* q_empty = bars + 3;    // [2]
  uint64_t* do_full = bars + 5;
  uint64_t* do_empty = bars + 6;
  uint64_t* s_full = bars + 7;
  uint64_t* s_free = bars + 8;
  uint64_t* dp_full = bars + 9;
  uint64_t* p_full = bars + 10;
  uint64_t* dv_done = bars + 11;
  uint64_t* ds_full = bars + 12;
  uint64_t* dq_full = bars + 13;
  uint64_t* dq_free = bars + 14;
  uint64_t* pds_free = bars + 15;
  uint64_t* kv_done = bars + 16;
  uint64_t* drain = bars + 17;
  uint64_t* stg_full = bars + 18;  // [2]
  uint64_t* stg_free = bars + 20;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = a.B * a.H;
  int kt, bh;
  grouped_item((int)blockIdx.x, BH, a.n_tiles, false, bh, kt);  // small key tiles have the most work
  const int b = bh / a.H, h = bh % a.H;
  const int krow0 = b * a.T + kt * 128;
  const int i0 = a.causal ? kt : 0;
  const int n_it = a.n_tiles - i0;

  if (threadIdx.x == 0) {
    mbar_init(bar_kv, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&stg_full[i], 128);
      mbar_init(&stg_free[i], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(dp_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dv_done, 1);
    mbar_init(ds_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(pds_free, 1);
    mbar_init(kv_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tR0 = tmem, tR1 = tmem + 128, tDV = tmem + 256, tDK = tmem + 384;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      uint32_t q_valid = 0, q_par = 0;
      bool do_pending = false;
      uint32_t do_par = 0;
      mbar_arrive_expect_tx(bar_kv, 2 * TILE);
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        tma_load_3d(sK + p * kPanel, &tmK, bar_kv, h * D + p * 64, krow0, 0);
        tma_load_3d(sV + p * kPanel, &tmV, bar_kv, h * D + p * 64, krow0, 0);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        const int bf = it & 1;
        const int qi = i0 + it;
        const int qrow = b * a.T + qi * 128;
        if (it >= 2 && !mbar_wait(&q_empty[bf], ((it - 2) >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        fa_stamp(a.trace, 3, it, 0);
        mbar_arrive_expect_tx(&q_full[bf], TILE + 2 * 512);
        q_valid |= 1u << bf;
        q_par = (q_par & ~(1u << bf)) | ((uint32_t)((it >> 1) & 1) << bf);
        bulk_load(sLse + bf * 128, a.lse + (long long)bh * a.T + qi * 128, 512, &q_full[bf]);
        bulk_load(sDv + bf * 128, a.dvec + (long long)bh * a.T + qi * 128, 512, &q_full[bf]);
#pragma unroll
        for (int p = 0; p < 2; ++p) tma_load_3d(sQ + bf * TILE + p * kPanel, &tmQ, &q_full[bf], h * D + p * 64, qrow, 0);
        if (it >= 1 && !mbar_wait(do_empty, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        fa_stamp(a.trace, 3, it, 1);
        mbar_arrive_expect_tx(do_full, TILE);
        do_pending = true;
        do_par = it & 1;
#pragma unroll
        for (int p = 0; p < 2; ++p) tma_load_3d(sDO + p * kPanel, &tmDO, do_full, h * D + p * 64, qrow, 0);
      }
      if (!ok) {
        *abort_flag = 1;
        const unsigned long long t0 = globaltimer_ns();
        for (int s = 0; s < 2; ++s) {
          if (!((q_valid >> s) & 1u)) continue;
          while (!mbar_try_wait(&q_full[s], (q_par >> s) & 1u))
            if (globaltimer_ns() - t0 > 100000000ull) break;
        }
        while (do_pending && !mbar_try_wait(do_full, do_par))
          if (globaltimer_ns() - t0 > 200000000ull) break;
        while (!mbar_try_wait(bar_kv, 0))
          if (globaltimer_ns() - t0 > 300000000ull) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // Order per query tile i: dP^T(i), dV(i), S^T(i+1), dQ(i), dK(i) -- S^T(i+1) goes out
    // before the wait for dS(i), so the softmax warps find it done when they move on and
    // compute P(i+1) while the tensor core runs dQ(i) and dK(i); dQ(i) goes first so that
    // its drain frees R1 for dP^T(i+1) while dK(i) still runs.
    if (lane == 0) {
      bool ok = mbar_wait(bar_kv, 0, abort_flag, a.err, ERR_TIMEOUT_MMA);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), pd_addr = smem_u32(sPD), do_addr = smem_u32(sDO);
      auto issue_s = [&](int it) -> bool {  // S^T(it) = K Q_it^T into R0
        if (!mbar_wait(&q_full[it & 1], (it >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) return false;
        if (it >= 1 && !mbar_wait(s_free, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + (it & 1) * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_bf16(tR0, desc_kmajor(k_addr, kk), desc_kmajor(q_addr, kk), IDESC_SS, kk > 0 ? 1u : 0u);
        umma_commit(s_full);
        return true;
      };
      if (ok && n_it > 0) ok = issue_s(0);
      for (int it = 0; it < n_it && ok; ++it) {
        const int bf = it & 1;
        const uint32_t q_addr = smem_u32(sQ + bf * TILE);
        fa_stamp(a.trace, 0, it, 4);
        if (!mbar_wait(do_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        fa_stamp(a.trace, 0, it, 5);
        if (it >= 1 && !mbar_wait(dq_free, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        fa_stamp(a.trace, 0, it, 6);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // dP^T = V dO^T
          umma_bf16(tR1, desc_kmajor(v_addr, kk), desc_kmajor(do_addr, kk), IDESC_SS, kk > 0 ? 1u : 0u);
        umma_commit(dp_full);
        fa_stamp(a.trace, 0, it, 0);
        if (!mbar_wait(p_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        fa_stamp(a.trace, 0, it, 1);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO, P^T from TMEM (over S^T's first 64 columns)
          umma_bf16_tmem_a(tDV, tR0 + kk * 8, desc_mnmajor(do_addr, kk), IDESC_KV, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(dv_done);
        umma_commit(do_empty);  // dO read by dP^T and dV
        if (it + 1 < n_it && !issue_s(it + 1)) { ok = false; break; }
        fa_stamp(a.trace, 0, it, 2);
        if (!mbar_wait(ds_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_MMA)) { ok = false; break; }
        fa_stamp(a.trace, 0, it, 3);
        tc_fence_after();
        // dQ first: its drain (and so the next dP^T, which reuses R1) starts while dK runs
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dQ = dS K  (into R1: dP^T has been read)
          umma_bf16(tR1, desc_mnmajor(pd_addr, kk), desc_mnmajor(k_addr, kk), IDESC_Q, kk > 0 ? 1u : 0u);
        umma_commit(dq_full);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dK += dS^T Q
          umma_bf16(tDK, desc_kmajor(pd_addr, kk), desc_mnmajor(q_addr, kk), IDESC_KV, (it > 0 || kk > 0) ? 1u : 0u);
        umma_commit(pds_free);
        umma_commit(&q_empty[bf]);
      }
      if (ok) {
        umma_commit(kv_done);
      } else {
        *abort_flag = 1;
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0))
          if (globaltimer_ns() - t0 > 100000000ull) break;
      }
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------------ P, dS, epilogue
    // Eight warps: two per TMEM lane quarter, each taking 64 of the row's 128 columns, so
    // every SM sub-partition runs two of them and their TMEM-load and MUFU latencies
    // overlap.  A thread's 64 columns are read with one wait; LSE is turned into
    // -LSE * log2(e) once per query tile and read with the Dvec terms as 16-byte
    // broadcasts; the math runs on packed fp32 pairs, and a quarter of the exponentials
    // on the FMA pipe (exp2_poly2).
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;  // columns [64 half, 64 half + 64)
    const int cb = half * 64;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float c = a.scale_log2;
    const float2 c2 = make_float2(c, c);
    bool ok = true;
    for (int it = 0; it < n_it; ++it) {
      const int bf = it & 1;
      const int i = i0 + it;
      float* nlse = sLse + bf * 128;
      const float* dvec = sDv + bf * 128;
      const bool stamp = warp == 2 && lane == 0;
      if (stamp) fa_stamp(a.trace, 1, it, 0);
      if (!mbar_wait_warp(&q_full[bf], (it >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (half == 0) nlse[r] = -nlse[r] * kLog2e;
      named_bar_sync(1, 256);
      if (!mbar_wait_warp(s_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (stamp) fa_stamp(a.trace, 1, it, 1);
      tc_fence_after();
      const bool diag = a.causal && (i == kt);
      uint32_t pk[32];  // this thread's 64 columns of the P^T row, packed bf16 pairs (kept for dS)
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t sv[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tR0 + lane_off + cb + h2 * 32, sv);
        tmem_ld_wait();
#pragma unroll
        for (int e0 = 0; e0 < 32; e0 += 4) {
          const int e = h2 * 32 + e0;
          const int cc = cb + e;
          const float4 n4 = *reinterpret_cast<const float4*>(nlse + cc);
          const float2 v0 = __ffma2_rn(make_float2(__uint_as_float(sv[e0]), __uint_as_float(sv[e0 + 1])), c2,
                                       make_float2(n4.x, n4.y));
          const float2 v1 = __ffma2_rn(make_float2(__uint_as_float(sv[e0 + 2]), __uint_as_float(sv[e0 + 3])), c2,
                                       make_float2(n4.z, n4.w));
          float2 p0, p1;
          if (e >= 48) {
            p0 = exp2_poly2(v0);
            p1 = exp2_poly2(v1);
          } else {
            p0 = make_float2(ex2_approx(v0.x), ex2_approx(v0.y));
            p1 = make_float2(ex2_approx(v1.x), ex2_approx(v1.y));
          }
          if (diag) {  // query cc precedes key r: no attention
            if (cc < r) p0.x = 0.f;
            if (cc + 1 < r) p0.y = 0.f;
            if (cc + 2 < r) p1.x = 0.f;
            if (cc + 3 < r) p1.y = 0.f;
          }
          pk[e >> 1] = pack_bf16x2(p0.x, p0.y);
          pk[(e >> 1) + 1] = pack_bf16x2(p1.x, p1.y);
        }
      }
      // P^T back into TMEM over the first 64 columns of S^T (this thread's 64 queries as 32
      // packed columns): the dV MMA reads it as its A operand, and S^T(i+1) is issued only
      // after that MMA (one thread's tcgen05 MMAs run in issue order)
      __syncwarp();
      tmem_st_32x32b_x32(tR0 + lane_off + half * 32, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(s_free);
      mbar_arrive(p_full);
      if (stamp) fa_stamp(a.trace, 1, it, 2);
      if (!mbar_wait_warp(dp_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (stamp) fa_stamp(a.trace, 1, it, 3);
      tc_fence_after();
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t dv[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tR1 + lane_off + cb + h2 * 32, dv);
        tmem_ld_wait();
#pragma unroll
        for (int e0 = 0; e0 < 32; e0 += 4) {
          const int e = h2 * 32 + e0;
          const int cc = cb + e;
          const float4 d4 = *reinterpret_cast<const float4*>(dvec + cc);
          const float2 pa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk[e >> 1]));
          const float2 pb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pk[(e >> 1) + 1]));
          const float2 da = __fadd2_rn(make_float2(__uint_as_float(dv[e0]), __uint_as_float(dv[e0 + 1])),
                                       make_float2(-d4.x, -d4.y));
          const float2 db = __fadd2_rn(make_float2(__uint_as_float(dv[e0 + 2]), __uint_as_float(dv[e0 + 3])),
                                       make_float2(-d4.z, -d4.w));
          const float2 sa = __fmul2_rn(pa, da), sb = __fmul2_rn(pb, db);
          pk[e >> 1] = pack_bf16x2(sa.x, sa.y);  // dS^T overwrites P^T in registers too
          pk[(e >> 1) + 1] = pack_bf16x2(sb.x, sb.y);
        }
      }
      if (stamp) fa_stamp(a.trace, 1, it, 4);
      // the dS tile is free once dQ(i-1) and dK(i-1) have read it
      if (it >= 1 && !mbar_wait_warp(pds_free, (it - 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (stamp) fa_stamp(a.trace, 1, it, 5);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        *reinterpret_cast<uint4*>(sPD + half * kPanel + sw128_chunk_offset(r, q)) =
            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      if (stamp) fa_stamp(a.trace, 1, it, 6);
    }
    if (ok && mbar_wait_warp(kv_done, 0, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      __nv_bfloat16* dvp = a.dV + (long long)(krow0 + r) * a.lddv + h * D + cb;
      __nv_bfloat16* dkp = a.dK + (long long)(krow0 + r) * a.lddk + h * D + cb;
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        uint32_t o[32];
        float f[32];
        __syncwarp();
        tmem_ld_32x32b_x32(tDV + lane_off + cb + cc * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 32; ++v) f[v] = __uint_as_float(o[v]);
        store_row_bf16_global(dvp + cc * 32, f, 32);
        __syncwarp();
        tmem_ld_32x32b_x32(tDK + lane_off + cb + cc * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int v = 0; v < 32; ++v) f[v] = __uint_as_float(o[v]) * a.scale;
        store_row_bf16_global(dkp + cc * 32, f, 32);
      }
    }
  } else {
    // ------------------------------------------------------------------ dQ drain (TMA reduce-add)
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const bool issuer = (warp == 10 && lane == 0);
    int g = 0;          // staging slices issued so far (this CTA)
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const int i = i0 + it;
      if (issuer) fa_stamp(a.trace, 2, it, 0);
      if (!mbar_wait_warp(dq_full, it & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (issuer) fa_stamp(a.trace, 2, it, 1);
      tc_fence_after();
      // two 64-column halves (64 registers); R1 is released once both have been read
#pragma unroll 1
      for (int hh = 0; hh < 2 && ok; ++hh) {
        uint32_t o[2][32];
        __syncwarp();
        tmem_ld_32x32b_x32(tR1 + lane_off + hh * 64, o[0]);
        tmem_ld_32x32b_x32(tR1 + lane_off + hh * 64 + 32, o[1]);
        tmem_ld_wait();
        if (hh == 1) {
          tc_fence_before();
          mbar_arrive(dq_free);  // R1 may take dP^T of the next tile
          if (issuer) fa_stamp(a.trace, 2, it, 2);
        }
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2, ++g) {
          const int cc = hh * 2 + c2;
          const int sb = g & 1;
          if (g >= 2 && !mbar_wait_warp(&stg_free[sb], ((g - 2) >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) {
            ok = false;
            break;
          }
          uint8_t* st = sDQ + sb * STG;
#pragma unroll
          for (int q = 0; q < 8; ++q) {  // row r: 32 fp32 = 8 x 16 B chunks, 128-byte swizzle
            const float4 v = make_float4(__uint_as_float(o[c2][4 * q]) * a.scale, __uint_as_float(o[c2][4 * q + 1]) * a.scale,
                                         __uint_as_float(o[c2][4 * q + 2]) * a.scale, __uint_as_float(o[c2][4 * q + 3]) * a.scale);
            *reinterpret_cast<float4*>(st + r * 128 + ((q ^ (r & 7)) << 4)) = v;
          }
          fence_proxy_async_smem();
          mbar_arrive(&stg_full[sb]);
          if (issuer) {
            if (!mbar_wait(&stg_full[sb], (g >> 1) & 1, abort_flag, a.err, ERR_TIMEOUT_EPILOGUE)) {
              ok = false;
            } else {
              tma_reduce_add_3d(&tmDQ, st, h * D + cc * 32, b * a.T + i * 128, 0);
              bulk_commit_group();
              if (g >= 1) {
                bulk_wait_group_read<1>();            // slice g-1 has been read from shared memory
                mbar_arrive(&stg_free[(g - 1) & 1]);
              }
            }
          }
          ok = __all_sync(0xffffffffu, ok) != 0;
          if (!ok) break;
        }
      }
    }
    if (issuer) bulk_wait_group<0>();  // every reduce-add has completed before the CTA exits
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Dvec[bh, t] = sum_d dO[t, h*D + d] * O[t, h*D + d]; one warp per (row, head).
__global__ void fa_bwd_dot_kernel(const __nv_bfloat16* __restrict__ dO, long long lddo,
                                  const __nv_bfloat16* __restrict__ O, long long ldo, float* __restrict__ dvec,
                                  int B, int T, int H, int D) {
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= (long long)B * T * H) return;
  const int row = (int)(w / H), h = (int)(w % H);
  const __nv_bfloat16* g = dO + (long long)row * lddo + h * D;
  const __nv_bfloat16* o = O + (long long)row * ldo + h * D;
  float acc = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const float2 gf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(g + d));
    const float2 of = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(o + d));
    acc += gf.x * of.x + gf.y * of.y;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    const int b = row / T, t = row % T;
    dvec[((long long)b * H + h) * T + t] = acc;
  }
}

// bf16 copy of an fp32 [rows, cols] accumulator into a strided bf16 destination.
__global__ void f32_to_bf16_rows_kernel(const float* __restrict__ src, long long lds, __nv_bfloat16* __restrict__ dst,
                                        long long ldd, int rows, int cols) {
  const long long idx = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const long long total = (long long)rows * cols;
  if (idx >= total) return;
  const int r = (int)(idx / cols), c = (int)(idx % cols);
  const float4 a = *reinterpret_cast<const float4*>(src + r * lds + c);
  const float4 bq = *reinterpret_cast<const float4*>(src + r * lds + c + 4);
  uint4 u;
  u.x = pack_bf16x2(a.x, a.y);
  u.y = pack_bf16x2(a.z, a.w);
  u.z = pack_bf16x2(bq.x, bq.y);
  u.w = pack_bf16x2(bq.z, bq.w);
  *reinterpret_cast<uint4*>(dst + r * ldd + c) = u;
}

// ------------------------------------------------------------------------------ host
template <typename K>
static void set_smem(K kern, size_t bytes) {
  C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
}

static void check_view(const torch::Tensor& t, const char* n, int64_t rows, int64_t cols) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2, n, ": CUDA bf16 2-D view");
  TORCH_CHECK(t.stride(1) == 1 && t.size(0) == rows && t.size(1) >= cols, n, ": [B*T, >= H*D] with unit inner stride");
  TORCH_CHECK((t.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, n, ": 16-byte aligned rows");
}

static long long* g_fa_trace = nullptr;

// Install (or with None remove) an int64 [4 * 64 * 8] buffer that the next flash-attention
// launches fill with the phase timeline of their CTA 0 (clock64 values).
void fa_trace_set(c10::optional<torch::Tensor> buf) {
  if (buf.has_value()) {
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kLong && buf->numel() >= 4 * 64 * 8, "int64 [2048]");
    g_fa_trace = reinterpret_cast<long long*>(buf->data_ptr<int64_t>());
  } else {
    g_fa_trace = nullptr;
  }
}

// q, k, v: [B*T, *] row views (head h at cols h*D); out: [B*T, >= H*D]; lse: fp32 [B*H*T]
void fa_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, int64_t B, int64_t T, int64_t H, int64_t D,
            double scale, bool causal, torch::Tensor out, torch::Tensor lse, torch::Tensor err) {
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(T % 128 == 0, "sequence length must be a multiple of 128");
  const int64_t rows = B * T, cols = H * D;
  check_view(q, "q", rows, cols);
  check_view(k, "k", rows, cols);
  check_view(v, "v", rows, cols);
  check_view(out, "out", rows, cols);
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() >= B * H * T, "lse fp32 [B*H*T]");
  c10::cuda::CUDAGuard guard(q.device());
  CUtensorMap tq = make_tmap_bf16(q.data_ptr(), cols, rows, q.stride(0), 64, 128, 1, 0);
  CUtensorMap tk = make_tmap_bf16(k.data_ptr(), cols, rows, k.stride(0), 64, 128, 1, 0);
  CUtensorMap tv = make_tmap_bf16(v.data_ptr(), cols, rows, v.stride(0), 64, 128, 1, 0);
  FaArgs a{};
  a.B = (int)B; a.T = (int)T; a.H = (int)H; a.n_tiles = (int)(T / 128); a.causal = causal ? 1 : 0;
  a.scale = (float)scale; a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.O = reinterpret_cast<__nv_bfloat16*>(out.data_ptr()); a.ldo = out.stride(0);
  a.lse = lse.data_ptr<float>();
  a.err = err.data_ptr<int>();
  a.trace = g_fa_trace;
  const unsigned grid = (unsigned)(B * H * (T / 128));
  auto s = at::cuda::getCurrentCUDAStream();
  static const bool one_tile = getenv("TFB_FA_FWD_ONE_TILE") != nullptr;
  if (D == 128 && T % 256 == 0 && !one_tile) {
    static bool init = false;
    if (!init) { set_smem(fa_fwd2_kernel, kFwd2Smem); init = true; }
    fa_fwd2_kernel<<<grid / 2, 320, kFwd2Smem, s>>>(tq, tk, tv, a);
  } else if (D == 128) {
    static bool init = false;
    if (!init) { set_smem(fa_fwd_kernel<128>, FaCfg<128>::FWD_SMEM); init = true; }
    fa_fwd_kernel<128><<<grid, 192, FaCfg<128>::FWD_SMEM, s>>>(tq, tk, tv, a);
  } else {
    static bool init = false;
    if (!init) { set_smem(fa_fwd_kernel<64>, FaCfg<64>::FWD_SMEM); init = true; }
    fa_fwd_kernel<64><<<grid, 192, FaCfg<64>::FWD_SMEM, s>>>(tq, tk, tv, a);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Gradients: dq_acc (fp32, zeroed here) accumulates dQ; dk / dv receive bf16 dK / dV;
// dq_out (bf16 view) receives dQ.  dvec: fp32 scratch [B*H*T].
void fa_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o, torch::Tensor dout, torch::Tensor lse,
            int64_t B, int64_t T, int64_t H, int64_t D, double scale, bool causal, torch::Tensor dq_acc,
            torch::Tensor dq_out, torch::Tensor dk, torch::Tensor dv, torch::Tensor dvec, torch::Tensor err) {
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(T % 128 == 0, "sequence length must be a multiple of 128");
  const int64_t rows = B * T, cols = H * D;
  check_view(q, "q", rows, cols);
  check_view(k, "k", rows, cols);
  check_view(v, "v", rows, cols);
  check_view(o, "o", rows, cols);
  check_view(dout, "dout", rows, cols);
  check_view(dk, "dk", rows, cols);
  check_view(dv, "dv", rows, cols);
  check_view(dq_out, "dq_out", rows, cols);
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.dim() == 2 && dq_acc.size(0) == rows &&
                  dq_acc.stride(1) == 1 && dq_acc.size(1) >= cols,
              "dq_acc fp32 [B*T, >= H*D]");
  c10::cuda::CUDAGuard guard(q.device());
  auto s = at::cuda::getCurrentCUDAStream();
  dq_acc.zero_();
  {
    const long long warps = rows * H;
    fa_bwd_dot_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0),
        reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), o.stride(0), dvec.data_ptr<float>(), (int)B, (int)T,
        (int)H, (int)D);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  CUtensorMap tq = make_tmap_bf16(q.data_ptr(), cols, rows, q.stride(0), 64, 128, 1, 0);
  CUtensorMap tk = make_tmap_bf16(k.data_ptr(), cols, rows, k.stride(0), 64, 128, 1, 0);
  CUtensorMap tv = make_tmap_bf16(v.data_ptr(), cols, rows, v.stride(0), 64, 128, 1, 0);
  CUtensorMap tdo = make_tmap_bf16(dout.data_ptr(), cols, rows, dout.stride(0), 64, 128, 1, 0);
  FaArgs a{};
  a.B = (int)B; a.T = (int)T; a.H = (int)H; a.n_tiles = (int)(T / 128); a.causal = causal ? 1 : 0;
  a.scale = (float)scale; a.scale_log2 = (float)(scale * 1.4426950408889634);
  a.lse = lse.data_ptr<float>();
  a.dvec = dvec.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>(); a.lddq = dq_acc.stride(0);
  a.dK = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()); a.lddk = dk.stride(0);
  a.dV = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()); a.lddv = dv.stride(0);
  a.err = err.data_ptr<int>();
  a.trace = g_fa_trace;
  const unsigned grid = (unsigned)(B * H * (T / 128));
  static const bool serial_bwd = getenv("TFB_FA_BWD_SERIAL") != nullptr;
  if (D == 128 && !serial_bwd) {
    static bool init = false;
    if (!init) { set_smem(fa_bwd2_kernel, kBwd2Smem); init = true; }
    CUtensorMap tdq = make_tmap_f32(dq_acc.data_ptr(), cols, rows, dq_acc.stride(0), 32, 128);
    fa_bwd2_kernel<<<grid, 448, kBwd2Smem, s>>>(tq, tk, tv, tdo, tdq, a);
  } else if (D == 128) {
    static bool init = false;
    if (!init) { set_smem(fa_bwd_kernel<128>, FaCfg<128>::BWD_SMEM); init = true; }
    fa_bwd_kernel<128><<<grid, 192, FaCfg<128>::BWD_SMEM, s>>>(tq, tk, tv, tdo, a);
  } else {
    static bool init = false;
    if (!init) { set_smem(fa_bwd_kernel<64>, FaCfg<64>::BWD_SMEM); init = true; }
    fa_bwd_kernel<64><<<grid, 192, FaCfg<64>::BWD_SMEM, s>>>(tq, tk, tv, tdo, a);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  {
    const long long n8 = rows * cols / 8;
    f32_to_bf16_rows_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(
        dq_acc.data_ptr<float>(), dq_acc.stride(0), reinterpret_cast<__nv_bfloat16*>(dq_out.data_ptr()),
        dq_out.stride(0), (int)rows, (int)cols);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace tfb
