// tcgen05 BF16 GEMM with fused epilogues for the encoder/head projections.
//
// Replaces the reference's cuBLAS `gemm_ex` calls (src/cuda/mod.rs:347-375)
// and the row kernels that consumed their BF16 outputs:
//   Wqkv                 -> EPI_QKV_ROPE (RoPE of src/cuda/kernels.cu:215-252 moved here)
//   Wi + geglu           -> EPI_GEGLU    (kernels.cu:137-155)
//   Wo / Wo2 + ln_bf16   -> EPI_RESID_LN (kernels.cu:97-109, residual added in FP32)
//   head in_proj/lin1    -> EPI_BF16 with bias (+relu)  (kernels.cu:158-172)
//   scorer W1 + scorer   -> EPI_SCORER   (kernels.cu:186-194)
//
// Structure: persistent CTAs (one per SM), 192 threads.
//   warp 0      TMA producer: A (128 x 64) and W (BN x 64) boxes into a smem ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16)
//   warps 2..5  epilogue: tcgen05.ld of the FP32 accumulator (lane = row), fused math,
//               direct global stores
// The accumulator is double buffered in TMEM (2 x BN columns) so the epilogue
// of one tile overlaps the main loop of the next.
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace j1rt {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;

template <int BN>
struct GemmCfg {
  static constexpr int STAGES = (BN == 256) ? 4 : 6;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

__device__ __forceinline__ void store_bf16x32(bf16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 q;
    q.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
    q.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    q.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    q.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    d[i] = q;
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const EpiParams p) {
  using C = GemmCfg<BN>;
  constexpr bool FULL_ROW = (EPI == EPI_RESID_LN || EPI == EPI_RESID || EPI == EPI_SCORER);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int m_tiles = (p.M + BM - 1) / BM;
  const int n_sub = FULL_ROW ? p.N / BN : 1;
  const int n_per_m = FULL_ROW ? 1 : p.N / BN;
  const int units = m_tiles * n_per_m;
  const int kblocks = p.K / BK;
  {  // exit before allocating anything when an earlier CTA of this launch gave up
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = device_aborted(p.err) ? 1 : 0;
    __syncthreads();
    if (s_abort) return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_par = 0;  // per stage: armed bit and the parity it was armed with
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int mt = u / n_per_m, nu = u % n_per_m;
        for (int s = 0; s < n_sub && ok; ++s) {
          const int n0 = (FULL_ROW ? s : nu) * BN;
          for (int kb = 0; kb < kblocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.err, 1)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
            tma_load_2d(&tmA, &full[stage], sA + stage * C::A_BYTES, kb * BK, mt * BM);
            tma_load_2d(&tmW, &full[stage], sB + stage * C::B_BYTES, kb * BK, n0);
            armed |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        // Unwinding: let every copy already in flight land before smem is released.
        volatile int no_abort = 0;
        for (int s = 0; s < C::STAGES; ++s)
          if (armed & (1u << s)) mbar_wait(&full[s], (armed_par >> s) & 1u, &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        for (int s = 0; s < n_sub && ok; ++s) {
          const int buf = acc & 1;
          const uint32_t aph = (acc >> 1) & 1;
          if (!mbar_wait(&tempty[buf], aph ^ 1, abort_flag, p.err, 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + buf * BN;
          for (int kb = 0; kb < kblocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, abort_flag, p.err, 3)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
            const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              umma_bf16(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                        (kb | k) != 0);
            }
            umma_commit(&empty[stage]);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit(&tfull[buf]);
          ++acc;
        }
      }
      // All MMAs of this thread must have finished before TMEM is released.
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int trow = q * 32 + lane;
    int acc = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int mt = u / n_per_m, nu = u % n_per_m;
      const int row = mt * BM + trow;
      const bool valid = row < p.M;
      float rsum = 0.f;   // full-row residual sum (LN mean)
      float score = 0.f;  // scorer dot product
      for (int s = 0; s < n_sub; ++s) {
        const int buf = acc & 1;
        const uint32_t aph = (acc >> 1) & 1;
        if (!mbar_wait(&tfull[buf], aph, abort_flag, p.err, 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
        const int n0 = (FULL_ROW ? s : nu) * BN;

        if constexpr (EPI == EPI_BF16) {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tb + c * 32, r);
            tmem_ld_wait();
            float v[32];
            const int col = n0 + c * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float a = __uint_as_float(r[j]);
              if (p.bias) a += p.bias[col + j];
              if (p.relu) a = fmaxf(a, 0.f);
              v[j] = a;
            }
            if (valid) store_bf16x32(p.out + static_cast<size_t>(row) * p.ldo + col, v);
          }
        } else if constexpr (EPI == EPI_QKV_ROPE) {
          const int ps = valid ? p.pos[row] : 0;
          const float* cs = p.rope_cos + static_cast<size_t>(ps) * 32;
          const float* sn = p.rope_sin + static_cast<size_t>(ps) * 32;
#pragma unroll 1
          for (int g = 0; g < BN / 64; ++g) {
            uint32_t lo[32], hi[32];
            tmem_ld32(tb + g * 64, lo);
            tmem_ld32(tb + g * 64 + 32, hi);
            tmem_ld_wait();
            const int col = n0 + g * 64;
            float a[32], b[32];
            if (col < p.rope_cols) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float x = __uint_as_float(lo[j]), y = __uint_as_float(hi[j]);
                const float c = cs[j], sv = sn[j];
                a[j] = x * c - y * sv;
                b[j] = y * c + x * sv;
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                a[j] = __uint_as_float(lo[j]);
                b[j] = __uint_as_float(hi[j]);
              }
            }
            if (valid) {
              bf16* dst = p.out + static_cast<size_t>(row) * p.ldo + col;
              store_bf16x32(dst, a);
              store_bf16x32(dst + 32, b);
            }
          }
        } else if constexpr (EPI == EPI_GEGLU) {
          static_assert(BN == 256, "GEGLU tiles hold 128 gate-input + 128 gate columns");
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t ra[32], rb[32];
            tmem_ld32(tb + c * 32, ra);
            tmem_ld32(tb + 128 + c * 32, rb);
            tmem_ld_wait();
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_erf(__uint_as_float(ra[j])) * __uint_as_float(rb[j]);
            if (valid) store_bf16x32(p.out + static_cast<size_t>(row) * p.ldo + nu * 128 + c * 32, v);
          }
        } else if constexpr (EPI == EPI_RESID_LN || EPI == EPI_RESID) {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tb + c * 32, r);
            tmem_ld_wait();
            const int col = n0 + c * 32;
            if (valid) {
              float4* xr = reinterpret_cast<float4*>(p.x + static_cast<size_t>(row) * p.ldx + col);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float4 o = xr[i];
                float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
                if (p.bias) {
                  b0 = p.bias[col + 4 * i];
                  b1 = p.bias[col + 4 * i + 1];
                  b2 = p.bias[col + 4 * i + 2];
                  b3 = p.bias[col + 4 * i + 3];
                }
                o.x += __uint_as_float(r[4 * i]) + b0;
                o.y += __uint_as_float(r[4 * i + 1]) + b1;
                o.z += __uint_as_float(r[4 * i + 2]) + b2;
                o.w += __uint_as_float(r[4 * i + 3]) + b3;
                xr[i] = o;
                rsum += (o.x + o.y) + (o.z + o.w);
              }
            }
          }
        } else if constexpr (EPI == EPI_SCORER) {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tb + c * 32, r);
            tmem_ld_wait();
            const int col = n0 + c * 32;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              score += gelu_erf(__uint_as_float(r[j]) + p.bias[col + j]) * p.w2[col + j];
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty[buf]);
        ++acc;
      }
      if (!ok) break;
      if constexpr (EPI == EPI_RESID_LN) {
        if (valid) {
          // Two-pass LayerNorm over the updated row (re-read from L1/L2).
          const float inv_n = 1.f / static_cast<float>(p.N);
          const float mean = rsum * inv_n;
          const float4* xr = reinterpret_cast<const float4*>(p.x + static_cast<size_t>(row) * p.ldx);
          float ss = 0.f;
          for (int i = 0; i < p.N / 4; ++i) {
            const float4 v = xr[i];
            const float a = v.x - mean, b = v.y - mean, c = v.z - mean, d = v.w - mean;
            ss += (a * a + b * b) + (c * c + d * d);
          }
          const float rstd = rsqrtf(ss * inv_n + p.ln_eps);
          uint2* dst = reinterpret_cast<uint2*>(p.xn + static_cast<size_t>(row) * p.ldxn);
          const float4* w4 = reinterpret_cast<const float4*>(p.ln_w);
          const float4* b4 = reinterpret_cast<const float4*>(p.ln_b);
          for (int i = 0; i < p.N / 4; ++i) {
            const float4 v = xr[i];
            const float4 g = w4[i];
            float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p.ln_b) b = b4[i];
            uint2 o;
            o.x = pack_bf16x2((v.x - mean) * rstd * g.x + b.x, (v.y - mean) * rstd * g.y + b.y);
            o.y = pack_bf16x2((v.z - mean) * rstd * g.z + b.z, (v.w - mean) * rstd * g.w + b.w);
            dst[i] = o;
          }
        }
      } else if constexpr (EPI == EPI_SCORER) {
        if (valid) p.scores[row] = score + p.b2;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * BN);
}

template <int BN, int EPI>
int launch_one(const CUtensorMap& tmA, const CUtensorMap& tmW, const EpiParams& p, int grid_limit,
               cudaStream_t stream) {
  static bool configured = false;  // per instantiation; attribute set is idempotent
  auto kern = gemm_tc_kernel<BN, EPI>;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<BN>::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
  constexpr bool FULL_ROW = (EPI == EPI_RESID_LN || EPI == EPI_RESID || EPI == EPI_SCORER);
  const int units = ((p.M + BM - 1) / BM) * (FULL_ROW ? 1 : p.N / BN);
  const int grid = units < grid_limit ? units : grid_limit;
  if (grid <= 0) return 0;
  kern<<<grid, 192, GemmCfg<BN>::SMEM, stream>>>(tmA, tmW, p);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace

int gemm_bn_for(int n) { return (n % 256 == 0) ? 256 : 128; }

const char* gemm_shape_error(GemmEpi epi, int bn, int M, int N, int K) {
  if (M < 0 || N <= 0 || K <= 0) return "GEMM dimensions must be positive";
  if (bn != 128 && bn != 256) return "GEMM tile width must be 128 or 256";
  if (K % BK != 0) return "GEMM K must be a multiple of 64";
  if (N % bn != 0) return "GEMM N must be a multiple of the tile width";
  if (epi == EPI_GEGLU && bn != 256) return "GEGLU epilogue needs 256-wide tiles";
  if (epi == EPI_QKV_ROPE && bn % 64 != 0) return "RoPE epilogue needs whole heads per tile";
  return nullptr;
}

int launch_gemm(GemmEpi epi, int bn, const CUtensorMap& tmA, const CUtensorMap& tmW, const EpiParams& p,
                int grid_limit, cudaStream_t stream) {
  if (p.M == 0) return 0;
#define J1_GEMM_CASE(E)                                                                  \
  case E:                                                                                \
    return bn == 256 ? launch_one<256, E>(tmA, tmW, p, grid_limit, stream)               \
                     : launch_one<128, E>(tmA, tmW, p, grid_limit, stream);
  switch (epi) {
    J1_GEMM_CASE(EPI_BF16)
    J1_GEMM_CASE(EPI_QKV_ROPE)
    J1_GEMM_CASE(EPI_RESID_LN)
    J1_GEMM_CASE(EPI_RESID)
    J1_GEMM_CASE(EPI_SCORER)
    case EPI_GEGLU:
      return launch_one<256, EPI_GEGLU>(tmA, tmW, p, grid_limit, stream);
  }
#undef J1_GEMM_CASE
  return static_cast<int>(cudaErrorInvalidValue);
}

// ------------------------------------------------------------------ TMA maps
namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}
}  // namespace

bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                    uint32_t box_rows, const char** why) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    if (why) *why = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  if (rows == 0) rows = 1;  // an empty operand is never loaded; keep the map encodable
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (why) *why = "cuTensorMapEncodeTiled failed (alignment or shape)";
    return false;
  }
  return true;
}

}  // namespace j1rt
