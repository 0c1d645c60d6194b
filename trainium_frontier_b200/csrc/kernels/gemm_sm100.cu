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
// CTA = 6 warps, one CTA per SM, grid = min(#tiles, #SMs), tiles strided over CTAs:
//   warp 0      TMA producer            (full[s] <- TMA bytes, waits empty[s])
//   warp 1      TMEM owner + MMA issuer (waits full[s], commits empty[s] / tfull[a])
//   warps 2..5  epilogue, one TMEM lane quarter each (waits tfull[a], arrives tempty[a])
// Tile 128 x BN x 64 (BN = 256 or 128), 4 or 6 pipeline stages.
//
// Epilogues (the fused ops the model needs):
//   EPI_BF16      D = bf16(alpha * acc (+ R))               linear, linear + residual
//   EPI_RELU2     D2 = bf16(acc) (pre-activation h), D = bf16(relu(h - tau)^2)
//   EPI_RELU2_BWD D = bf16(bf16(alpha * acc) * 2 relu(R - tau))   (R = h)
//   EPI_F32       D(f32) = alpha * acc (+ D if beta)        weight gradients (fp32, split-K via
//                                                          vector atomics into the gradient)
// Every TMA load is a plain per-CTA load of this GPU's own memory.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "sm100_common.cuh"

namespace tfb {

enum GemmEpi : int { EPI_BF16 = 0, EPI_RELU2 = 1, EPI_RELU2_BWD = 2, EPI_F32 = 3 };

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
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128, BK = 64;
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + (2 * STAGES + 5) * 8 + 16;
};

__device__ __forceinline__ void decode_tile(int t, const GemmArgs& a, int& mb, int& nb, int& ks, int& bi) {
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

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmArgs args) {
  using C = GemmCfg<BN>;
  constexpr int BM = C::BM, BK = C::BK, STAGES = C::STAGES;
  constexpr uint32_t IDESC = umma_idesc_bf16(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * C::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t out_valid = 0, out_parity = 0;  // per-stage: a load is in flight / its phase parity
      for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x) {
        int mb, nb, ks, bi;
        decode_tile(t, args, mb, nb, ks, bi);
        const int kb0 = ks * args.kb_per_split;
        const int kb1 = min(kb0 + args.kb_per_split, args.kb_total);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.err, ERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES + C::B_BYTES);
          out_valid |= 1u << stage;
          out_parity = (out_parity & ~(1u << stage)) | (phase << stage);
          uint8_t* a_dst = sA + stage * C::A_BYTES;
          uint8_t* b_dst = sB + stage * C::B_BYTES;
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
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.num_tiles && ok; t += gridDim.x) {
        int mb, nb, ks, bi;
        decode_tile(t, args, mb, nb, ks, bi);
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
            umma_bf16(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);  // stage is free once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);  // accumulator ready for the epilogue
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        // Let every MMA already issued finish before TMEM is released.
        umma_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (globaltimer_ns() - t0 > 100000000ull) break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const float alpha = args.alpha * (args.alpha_ptr ? *args.alpha_ptr : 1.f);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x) {
      int mb, nb, ks, bi;
      decode_tile(t, args, mb, nb, ks, bi);
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, args.err, ERR_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const int row = mb * BM + q * 32 + lane;
      const bool row_ok = row < args.M;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
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
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
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

// 2-D bf16 tensor map with 128-byte swizzle.  inner/outer are element extents,
// row_stride_elems the distance between consecutive outer indices.
CUtensorMap make_tmap_bf16(const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                           uint32_t box_inner, uint32_t box_outer, uint64_t batch, uint64_t batch_stride_elems) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  TORCH_CHECK(batch == 1 || (batch_stride_elems * 2) % 16 == 0, "TMA batch stride must be a multiple of 16 bytes");
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

int num_sms(int dev) {
  static int cache[64] = {0};
  if (!cache[dev]) {
    cudaDeviceProp prop;
    C10_CUDA_CHECK(cudaGetDeviceProperties(&prop, dev));
    cache[dev] = prop.multiProcessorCount;
  }
  return cache[dev];
}

template <int BN, bool A_MN, bool B_MN, int EPI>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& a, int grid,
                        cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set = false;  // one per instantiation
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_set = true;
  }
  kern<<<grid, 192, C::SMEM, stream>>>(ta, tb, a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN>
static void dispatch(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                     const GemmArgs& a, int grid, cudaStream_t s) {
#define TFB_CASE(AM, BM_, E) \
  if (a_mn == AM && b_mn == BM_ && epi == E) return launch_gemm<BN, AM, BM_, E>(ta, tb, a, grid, s);
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
#undef TFB_CASE
  TORCH_CHECK(false, "unsupported gemm variant a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

// A: if !a_mn a [M, K] view (row stride lda), else a [K, M] view.  B likewise with N.
// Operands are 2-D, or 3-D with a leading batch dimension (all of A, B, D batched alike).
void gemm_bf16(torch::Tensor A, bool a_mn, torch::Tensor B, bool b_mn, int64_t M, int64_t N, int64_t K,
               torch::Tensor D, int64_t epi, double alpha, double beta, c10::optional<torch::Tensor> R,
               c10::optional<torch::Tensor> D2, double tau, int64_t split_k, int64_t bn, torch::Tensor err,
               c10::optional<torch::Tensor> alpha_t, double rcoef) {
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
  CUtensorMap ta = !a_mn ? make_tmap_bf16(A.data_ptr(), K, M, A.stride(0), 64, BM, nb, a_bs)
                         : make_tmap_bf16(A.data_ptr(), M, K, A.stride(0), 64, 64, nb, a_bs);
  CUtensorMap tb = !b_mn ? make_tmap_bf16(B.data_ptr(), K, N, B.stride(0), 64, (uint32_t)bn, nb, b_bs)
                         : make_tmap_bf16(B.data_ptr(), N, K, B.stride(0), 64, 64, nb, b_bs);
  GemmArgs a{};
  a.M = (int)M; a.N = (int)N; a.K = (int)K;
  a.tiles_m = (int)((M + BM - 1) / BM);
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
  const int grid = std::min(a.num_tiles, num_sms(A.get_device()));
  cudaStream_t s = at::cuda::getCurrentCUDAStream();
  if (bn == 256) dispatch<256>(a_mn, b_mn, (int)epi, ta, tb, a, grid, s);
  else dispatch<128>(a_mn, b_mn, (int)epi, ta, tb, a, grid, s);
}

}  // namespace tfb
