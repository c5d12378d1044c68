// tcgen05 BF16 GEMM with fused epilogues for the encoder/head projections.
//
// Replaces the reference's cuBLAS `gemm_ex` calls (src/cuda/mod.rs:347-375)
// and the row kernels that consumed their BF16 outputs:
//   Wqkv                 -> EPI_QKV_ROPE (RoPE of src/cuda/kernels.cu:215-252 moved here)
//   Wi + geglu           -> EPI_GEGLU    (kernels.cu:137-155)
//   head in_proj/lin1    -> EPI_BF16 with bias (+relu)  (kernels.cu:158-172)
//   scorer W1 + scorer   -> EPI_SCORER   (kernels.cu:186-194)
// (Wo / Wo2 with the residual and LayerNorm epilogues live in gemm_resid.cu.)
// Where the reference rounds a GEMM output to BF16 before a row kernel reads it (the QKV
// output before RoPE, both GEGLU halves), the epilogue rounds the FP32 accumulator at the
// same point.
//
// Structure: persistent CTA pairs (clusters of two CTAs on two SMs), 192 threads per CTA;
// the pair shares each 256-row tile through tcgen05 .cta_group::2 (see gemm_tc_kernel).
//   warp 0      TMA producer: A (128 x 64) and W (BN x 64) boxes into a smem ring
//   warp 1      TMEM allocator; in the even CTA also the single-thread tcgen05.mma issuer
//               (M=256 over the pair, N=BN, K=16)
//   warps 2..5  epilogue: tcgen05.ld of the FP32 accumulator (TMEM lane = row), fused math
// The accumulator is double buffered in TMEM (2 x BN columns) so the epilogue of one
// tile overlaps the main loop of the next.
//
// BF16 outputs (BF16, QKV_ROPE, GEGLU) are written row-per-thread into 128 x 64
// 128B-swizzled smem boxes (three in rotation) and leave by TMA store, so global
// writes are whole lines instead of 16-byte pieces of 32 different rows.
//
// The scorer epilogue owns whole rows: one work unit is 128 rows x H columns, computed as
// H/BN sub-tiles.
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace j1rt {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr uint32_t OBUF = 128 * 64 * 2;    // one 128-row x 64-column BF16 output box

__host__ __device__ constexpr bool is_full_row(int epi) { return epi == EPI_SCORER; }
__host__ __device__ constexpr bool is_tile_out(int epi) {
  return epi == EPI_BF16 || epi == EPI_QKV_ROPE || epi == EPI_GEGLU;
}

template <int BN, int EPI>
struct GemmCfg {
  // per CTA of a pair: 128 rows of A and BN/2 rows of W per stage; the ring takes what is
  // left of 227 KB after the output boxes
  static constexpr int STAGES = (EPI == EPI_SCORER) ? (BN == 256 ? 6 : 8) : (BN == 256 ? 5 : 7);
  static constexpr int THREADS = 192;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t O_BYTES = is_tile_out(EPI) ? 3 * OBUF : 0;
  static constexpr uint32_t SMEM =
      STAGES * STAGE_BYTES + O_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert((2 * STAGES + 5) * 8 + 8 <= 256, "barrier area");
};

__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }

// GEGLU outputs gelu(h0) * g0 and gelu(h1) * g1, evaluated pairwise with packed FP32
// arithmetic. erf(x) uses the rational approximation of the reference's CPU path
// (src/cpu/fastmath.rs:27-43; the Eigen/XLA float erf): x clamped to [-4, 4],
// erf = x p(x^2) / q(x^2) with p of degree 6 and q of degree 4 in x^2. Here x = h / sqrt(2)
// is folded into the coefficients (the clamp becomes |h| <= 4 sqrt(2), coefficient k of p
// and q is scaled by 2^-k, and p additionally by 1 / sqrt(2)), which saves the scaling of h;
// the division is a reciprocal estimate (about 1 ulp). It agrees with erff to about 1.2e-7,
// far below the BF16 rounding of the output.
__device__ __forceinline__ void geglu2(float h0, float h1, float g0, float g1, float& o0, float& o1) {
  constexpr float kClamp = 5.656854f;  // 4 sqrt(2)
  const uint64_t hc = f2pack(fminf(fmaxf(h0, -kClamp), kClamp), fminf(fmaxf(h1, -kClamp), kClamp));
  const uint64_t t = mul2(hc, hc);
  auto c2 = [](float c) { return f2pack(c, c); };
  uint64_t p = c2(-3.01199018e-12f);
  p = fma2(p, t, c2(6.1223987e-10f));
  p = fma2(p, t, c2(-9.28530142e-08f));
  p = fma2(p, t, c2(-5.03151205e-06f));
  p = fma2(p, t, c2(-0.00012992922f));
  p = fma2(p, t, c2(-0.00104460877f));
  p = fma2(p, t, c2(-0.011381614f));
  uint64_t q = c2(-9.10379526e-07f);
  q = fma2(q, t, c2(-2.6671758e-05f));
  q = fma2(q, t, c2(-0.000420706754f));
  q = fma2(q, t, c2(-0.00368666439f));
  q = fma2(q, t, c2(-0.01426474f));
  float q0, q1;
  f2unpack(q, q0, q1);
  const uint64_t erf = mul2(mul2(hc, p), f2pack(rcp_approx(q0), rcp_approx(q1)));
  const uint64_t hh = mul2(f2pack(h0, h1), c2(0.5f));
  f2unpack(mul2(fma2(hh, erf, hh), f2pack(g0, g1)), o0, o1);
}

// 32 values of one row -> four 16-byte units (unit0 .. unit0+3) of a 128B-swizzled box
// row: unit i of row r sits at (i ^ (r & 7)) * 16 within the row's 128 bytes.
__device__ __forceinline__ void put_row32(uint8_t* srow, int r, int unit0, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 q;
    q.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
    q.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    q.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    q.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    *reinterpret_cast<uint4*>(srow + ((static_cast<uint32_t>(unit0 + i) ^ (r & 7)) << 4)) = q;
  }
}

// BN: MMA tile width; NSUB: sub-tiles per full-row (scorer) unit (H = NSUB * BN).
// Launched as clusters of two CTAs (a pair). A pair computes 256-row tiles: each CTA
// loads its own 128 rows of A and its own half (BN/2 rows) of the W tile into smem, the
// even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = BN) over both CTAs' operands,
// and each CTA's TMEM receives the accumulator of its 128 rows, which its own epilogue
// warps consume. Per 128 x BN of output a CTA thus moves A + W/2 instead of A + W.
template <int BN, int EPI, int NSUB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GemmCfg<BN, EPI>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                   const __grid_constant__ CUtensorMap tmX, const EpiParams p) {
  using C = GemmCfg<BN, EPI>;
  constexpr bool FULL_ROW = is_full_row(EPI);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint8_t* sO = sB + C::STAGES * C::B_BYTES;  // 3 x OBUF output boxes when tile-out
  uint64_t* full = reinterpret_cast<uint64_t*>(sO + C::O_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  grid_dep_launch();
  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();  // 0: the CTA that issues the pair's MMAs
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int m_tiles = (p.M + 2 * BM - 1) / (2 * BM);
  const int n_sub = FULL_ROW ? NSUB : 1;
  const int n_per_m = FULL_ROW ? 1 : p.N / BN;
  const int units = m_tiles * n_per_m;
  const int kblocks = p.K / BK;
  {  // exit before allocating anything when an earlier CTA of this launch gave up; the
     // leader decides for both CTAs so that the pair stays together
    __shared__ int s_abort;
    if (leader && threadIdx.x == 0) {
      const int a = device_aborted(p.err) ? 1 : 0;
      s_abort = a;
      st_shared_cluster_u32(mapa_shared(smem_u32(&s_abort), 1), static_cast<uint32_t>(a));
    }
    cluster_sync();
    if (s_abort) return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW);
    if (is_tile_out(EPI)) tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  grid_dep_wait();  // the previous kernel's outputs (this kernel's inputs and outputs) are ready
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        const int mt = u / n_per_m, nu = u % n_per_m;
        const int m0 = mt * 2 * BM + static_cast<int>(rank) * BM;
        for (int s = 0; s < n_sub && ok; ++s) {
          const int n0 = (FULL_ROW ? s : nu) * BN + static_cast<int>(rank) * (BN / 2);
          for (int kb = 0; kb < kblocks; ++kb) {
            if (!mbar_wait<true>(&empty[stage], phase ^ 1, abort_flag, p.err, 1)) {
              ok = false;
              break;
            }
            // both CTAs' boxes of this stage complete on the leader's barrier
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_2d_pair(&tmA, fb, sA + stage * C::A_BYTES, kb * BK, m0);
            tma_load_2d_pair(&tmW, fb, sB + stage * C::B_BYTES, kb * BK, n0);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
      }
      if (!ok) {
        // Unwinding: loads of this CTA may complete on the other CTA's barrier, so they
        // cannot all be waited for here; give any copy in flight ample time to land
        // before the CTA releases its shared memory (this path only follows a timeout).
        const long long t0 = clock64();
        while (clock64() - t0 < 2000000) __nanosleep(1000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(2 * BM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        for (int s = 0; s < n_sub && ok; ++s) {
          const int buf = acc & 1;
          const uint32_t aph = (acc >> 1) & 1;
          if (!mbar_wait<true>(&tempty[buf], aph ^ 1, abort_flag, p.err, 2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + buf * BN;
          for (int kb = 0; kb < kblocks; ++kb) {
            if (!mbar_wait<true>(&full[stage], phase, abort_flag, p.err, 3)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
            const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              umma_bf16_pair(d, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024), idesc,
                             (kb | k) != 0);
            }
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&tfull[buf]), 1));
          ++acc;
        }
      }
      // All MMAs of this thread must have finished before TMEM is released (in both CTAs).
      umma_commit_pair(mapa_shared(smem_u32(drain), 0));
      volatile int no_abort = 0;
      mbar_wait<true>(drain, 0, &no_abort, nullptr, 0);
    }
  } else if (warp <= 5) {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    // Control flow is uniform across the 128 epilogue threads (named barriers below):
    // after an abort every wait returns at once and the loops run out without work.
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int trow = q * 32 + lane;
    const bool storer = (threadIdx.x == 64);  // issues the TMA stores of the epilogue
    int acc = 0;
    int ob = 0;        // output box in use (of three)
    // BF16 output: this thread's 64 values of row trow -> box `ob` (128B swizzle), then
    // one TMA store of the 128 x 64 box at (col, m0). Three boxes rotate: after issuing
    // a store the storer waits until only that store may still read smem, so the box
    // written next-but-one is free before any thread passes the next barrier.
    auto store_box = [&](const float (&a)[32], const float (&b)[32], int col, int m0) {
      uint8_t* srow = sO + ob * OBUF + trow * 128;
      put_row32(srow, trow, 0, a);
      put_row32(srow, trow, 4, b);
      fence_proxy_async_smem();
      named_bar_sync(1, 128);
      if (storer && !*abort_flag) {
        tma_store_2d(&tmX, sO + ob * OBUF, col, m0);
        bulk_commit();
        bulk_wait_read_1();
      }
      ob = (ob == 2) ? 0 : ob + 1;
    };
    for (int u = pair; u < units; u += npairs) {
      const int mt = u / n_per_m, nu = u % n_per_m;
      const int m0 = mt * 2 * BM + static_cast<int>(rank) * BM;  // this CTA's 128 rows
      const int row = m0 + trow;
      const bool valid = row < p.M;
      float score = 0.f;
      float4 rc[8], rsn[8];  // RoPE cos/sin of this row's position (QKV epilogue)
      if constexpr (EPI == EPI_QKV_ROPE) {
        const int ps = valid ? p.pos[row] : 0;
        const float4* c4 = reinterpret_cast<const float4*>(p.rope_cos + static_cast<size_t>(ps) * 32);
        const float4* s4 = reinterpret_cast<const float4*>(p.rope_sin + static_cast<size_t>(ps) * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          rc[i] = c4[i];
          rsn[i] = s4[i];
        }
      }
      for (int s = 0; s < n_sub; ++s) {
        const int buf = acc & 1;
        const uint32_t aph = (acc >> 1) & 1;
        mbar_wait<true>(&tfull[buf], aph, abort_flag, p.err, 4);
        tc_fence_after();
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
        const int n0 = (FULL_ROW ? s : nu) * BN;

        if constexpr (EPI == EPI_BF16) {
#pragma unroll 1
          for (int g = 0; g < BN / 64; ++g) {
            uint32_t lo[32], hi[32];
            tmem_ld32(tb + g * 64, lo);
            tmem_ld32(tb + g * 64 + 32, hi);
            tmem_ld_wait();
            const int col = n0 + g * 64;
            float a[32], b[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x = __uint_as_float(lo[j]), y = __uint_as_float(hi[j]);
              if (p.bias) {
                x += p.bias[col + j];
                y += p.bias[col + 32 + j];
              }
              if (p.relu) {
                x = fmaxf(x, 0.f);
                y = fmaxf(y, 0.f);
              }
              a[j] = x;
              b[j] = y;
            }
            store_box(a, b, col, m0);
          }
        } else if constexpr (EPI == EPI_QKV_ROPE) {
#pragma unroll 1
          for (int g = 0; g < BN / 64; ++g) {
            uint32_t lo[32], hi[32];
            tmem_ld32(tb + g * 64, lo);
            tmem_ld32(tb + g * 64 + 32, hi);
            tmem_ld_wait();
            const int col = n0 + g * 64;
            float a[32], b[32];
            if (col < p.rope_cols) {
              // qkv = bf16(acc) as the reference's GEMM writes it, then rotate-half on pairs
              // of dimensions at once (packed FP32):
              //   a = x c - y s,  b = y c + x s   for x = q[d], y = q[d + 32]
#pragma unroll
              for (int i = 0; i < 8; ++i) {
#pragma unroll
                for (int k = 0; k < 4; k += 2) {
                  const int j = 4 * i + k;
                  const uint64_t cc = k == 0 ? f2pack(rc[i].x, rc[i].y) : f2pack(rc[i].z, rc[i].w);
                  const uint64_t ss = k == 0 ? f2pack(rsn[i].x, rsn[i].y) : f2pack(rsn[i].z, rsn[i].w);
                  const uint64_t ns = k == 0 ? f2pack(-rsn[i].x, -rsn[i].y) : f2pack(-rsn[i].z, -rsn[i].w);
                  float x0 = __uint_as_float(lo[j]), x1 = __uint_as_float(lo[j + 1]);
                  float y0 = __uint_as_float(hi[j]), y1 = __uint_as_float(hi[j + 1]);
                  bf16_round2(x0, x1);
                  bf16_round2(y0, y1);
                  const uint64_t x = f2pack(x0, x1), y = f2pack(y0, y1);
                  f2unpack(fma2(y, ns, mul2(x, cc)), a[j], a[j + 1]);
                  f2unpack(fma2(x, ss, mul2(y, cc)), b[j], b[j + 1]);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                a[j] = __uint_as_float(lo[j]);
                b[j] = __uint_as_float(hi[j]);
              }
            }
            store_box(a, b, col, m0);
          }
        } else if constexpr (EPI == EPI_GEGLU) {
          static_assert(BN == 256, "GEGLU tiles hold 128 gate-input + 128 gate columns");
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float a[32], b[32];
            {
              uint32_t ra[32], rb[32];
              tmem_ld32(tb + h * 64, ra);
              tmem_ld32(tb + 128 + h * 64, rb);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; j += 2) {  // h = bf16(xn . Wi^T) as in the reference, then GEGLU
                float h0 = __uint_as_float(ra[j]), h1 = __uint_as_float(ra[j + 1]);
                float g0 = __uint_as_float(rb[j]), g1 = __uint_as_float(rb[j + 1]);
                bf16_round2(h0, h1);
                bf16_round2(g0, g1);
                geglu2(h0, h1, g0, g1, a[j], a[j + 1]);
              }
            }
            {
              uint32_t ra[32], rb[32];
              tmem_ld32(tb + h * 64 + 32, ra);
              tmem_ld32(tb + 128 + h * 64 + 32, rb);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 32; j += 2) {
                float h0 = __uint_as_float(ra[j]), h1 = __uint_as_float(ra[j + 1]);
                float g0 = __uint_as_float(rb[j]), g1 = __uint_as_float(rb[j + 1]);
                bf16_round2(h0, h1);
                bf16_round2(g0, g1);
                geglu2(h0, h1, g0, g1, b[j], b[j + 1]);
              }
            }
            store_box(a, b, nu * 128 + h * 64, m0);
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
        // this warp has read its lanes of the buffer: release it to the leader's MMA
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&tempty[buf]), 0));
        ++acc;
      }
      if constexpr (EPI == EPI_SCORER) {
        if (valid) p.scores[row] = score + p.b2;
      }
    }
    if (storer) bulk_wait_all();  // no store of ours may still read smem at exit
  }

  tc_fence_before();
  cluster_sync();  // every role of both CTAs is done and the leader's MMAs have drained
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, 2 * BN);
}

template <int BN, int EPI, int NSUB>
int launch_one(const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmX, const EpiParams& p,
               int grid_limit, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};  // per instantiation, one bit per device
  auto kern = gemm_tc_kernel<BN, EPI, NSUB>;
  const cudaError_t e = set_smem_once(kern, GemmCfg<BN, EPI>::SMEM, configured);
  if (e != cudaSuccess) return static_cast<int>(e);
  // work units are 256-row tiles of CTA pairs; grid_limit counts CTAs (SMs)
  const int units = ((p.M + 2 * BM - 1) / (2 * BM)) * (is_full_row(EPI) ? 1 : p.N / BN);
  const int max_pairs = grid_limit / 2 > 0 ? grid_limit / 2 : 1;
  const int pairs = units < max_pairs ? units : max_pairs;
  if (pairs <= 0) return 0;
  return static_cast<int>(
      launch_kernel(kern, dim3(2 * pairs), dim3(GemmCfg<BN, EPI>::THREADS), GemmCfg<BN, EPI>::SMEM, stream, tmA, tmW, tmX, p));
}

template <int EPI>
int launch_full_row(int H, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmX,
                    const EpiParams& p, int grid_limit, cudaStream_t stream) {
  switch (H) {
    case 256: return launch_one<256, EPI, 1>(tmA, tmW, tmX, p, grid_limit, stream);
    case 384: return launch_one<128, EPI, 3>(tmA, tmW, tmX, p, grid_limit, stream);
    case 512: return launch_one<256, EPI, 2>(tmA, tmW, tmX, p, grid_limit, stream);
    case 768: return launch_one<256, EPI, 3>(tmA, tmW, tmX, p, grid_limit, stream);
    case 1024: return launch_one<256, EPI, 4>(tmA, tmW, tmX, p, grid_limit, stream);
  }
  return static_cast<int>(cudaErrorInvalidValue);
}

}  // namespace

int gemm_bn_for(int n) { return (n % 256 == 0) ? 256 : 128; }

const char* gemm_shape_error(GemmEpi epi, int bn, int M, int N, int K) {
  if (M < 0 || N <= 0 || K <= 0) return "GEMM dimensions must be positive";
  if (bn != 128 && bn != 256) return "GEMM tile width must be 128 or 256";
  if (K % BK != 0) return "GEMM K must be a multiple of 64";
  if (N % bn != 0) return "GEMM N must be a multiple of the tile width";
  if (epi == EPI_GEGLU && bn != 256) return "GEGLU epilogue needs 256-wide tiles";
  const bool full_row = epi == EPI_RESID_LN || epi == EPI_RESID || epi == EPI_SCORER;
  if (full_row && !(N == 256 || N == 384 || N == 512 || N == 768 || N == 1024))
    return "full-row epilogues support N in {256, 384, 512, 768, 1024}";
  return nullptr;
}

int launch_gemm(GemmEpi epi, int bn, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap* tmX,
                const EpiParams& p, int grid_limit, cudaStream_t stream, const CUtensorMap* tmXs,
                const CUtensorMap* tmXN) {
  if (p.M == 0) return 0;
  if (!tmX && epi != EPI_SCORER) return static_cast<int>(cudaErrorInvalidValue);
  if (epi == EPI_RESID_LN || epi == EPI_RESID)
    return launch_resid_gemm(epi == EPI_RESID_LN, tmA, tmW, *tmX, tmXs, tmXN, p, grid_limit, stream);
  const CUtensorMap& X = tmX ? *tmX : tmA;  // unused by the scorer epilogue
  switch (epi) {
    case EPI_BF16:
      return bn == 256 ? launch_one<256, EPI_BF16, 1>(tmA, tmW, X, p, grid_limit, stream)
                       : launch_one<128, EPI_BF16, 1>(tmA, tmW, X, p, grid_limit, stream);
    case EPI_QKV_ROPE:
      return bn == 256 ? launch_one<256, EPI_QKV_ROPE, 1>(tmA, tmW, X, p, grid_limit, stream)
                       : launch_one<128, EPI_QKV_ROPE, 1>(tmA, tmW, X, p, grid_limit, stream);
    case EPI_GEGLU:
      return launch_one<256, EPI_GEGLU, 1>(tmA, tmW, X, p, grid_limit, stream);
    case EPI_SCORER:
      return launch_full_row<EPI_SCORER>(p.N, tmA, tmW, X, p, grid_limit, stream);
    default:
      break;
  }
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

bool make_tmap(CUtensorMap* map, CUtensorMapDataType dt, uint32_t esize, const void* base, uint64_t rows,
               uint64_t cols, uint64_t ld, uint32_t box_cols, uint32_t box_rows, const char** why) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    if (why) *why = "cuTensorMapEncodeTiled unavailable";
    return false;
  }
  if (rows == 0) rows = 1;  // an empty operand is never loaded; keep the map encodable
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * esize};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (why) *why = "cuTensorMapEncodeTiled failed (alignment or shape)";
    return false;
  }
  return true;
}
}  // namespace

bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                    uint32_t box_rows, const char** why) {
  return make_tmap(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, cols, ld, 64, box_rows, why);
}

bool make_tmap_f32_resid(CUtensorMap* map, const float* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         const char** why, uint32_t box_rows) {
  return make_tmap(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, rows, cols, ld, 32, box_rows, why);
}

}  // namespace j1rt
