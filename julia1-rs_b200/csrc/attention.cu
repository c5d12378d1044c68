// Varlen FlashAttention-style kernel on tcgen05 / TMEM for head_dim 64.
//
// Replaces the reference's mma.sync kernel `attention_impl` (src/cuda/kernels.cu:272-391)
// with the same semantics: packed sequences without padding, online softmax in base 2
// with scale 0.125*log2(e), an optional |i - j| <= window band (local layers,
// kernels.cu:304-308,332), and P rounded to BF16 before P.V. RoPE is not applied here:
// the Wqkv GEMM epilogue already rotated q and k.
//
// Work item = one 128-query tile of one sequence x one head. The kernel is persistent
// with two CTAs per SM (their pipelines interleave: one CTA's softmax overlaps the
// other's MMAs and loads); each CTA walks items blockIdx.x, +gridDim.x, ... with
// barriers, TMEM and smem set up once. 192 threads per CTA:
//   warps 0..3  softmax: thread r owns query row r (TMEM lane r); reads S from TMEM,
//               writes P (bf16 pairs) back to TMEM; O accumulates in TMEM over key blocks
//   warp 4      tcgen05.mma issuer: S = Q K^T (M=128, N=128, K=64, operands in smem) and
//               O += P V (M=128, N=64, K=128; P from TMEM, V from smem read MN-major)
//   warp 5      TMA producer: Q (double buffered across items), K/V blocks of 128 keys
//               (two stages)
// TMEM (256 columns): S [0,128), P [128,192) as packed bf16 pairs, O [192,256).
//
// Softmax: the first key block of an item computes the row max before the
// exponentials; later blocks exponentiate with the running offset while tracking the
// block max, and redo the block (and rescale O) only when the max grew by more than
// 2^8. P <= 2^8 then, and BF16 rounding of P is relative, so results match the
// always-rescaled online softmax to rounding.
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace j1rt {

namespace {

constexpr int QT = 128;   // queries per tile
constexpr int KB = 128;   // keys per block
constexpr int HD = 64;    // head dim
constexpr uint32_t TILE_BYTES = 128 * HD * 2;  // 16 KB per Q/K/V box
constexpr uint32_t ATT_SMEM = 6 * TILE_BYTES + 1024 + 256;  // Q x2, K x2, V x2
constexpr uint32_t TS_COL = 0, TP_COL = 128, TO_COL = 192;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A bounded wait whose outcome is the same in every lane of the warp: the softmax warps
// follow it with warp-collective tcgen05.ld/st, which all 32 lanes must reach together.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int site) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err, site));
}

// O (+)= P.V with P read from TMEM (A operand, K-major, two bf16 per 32-bit column).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Geometry of one work item (identical in every role of the CTA).
struct Item {
  AttnTile tl;
  int head, kbeg, nb;
};

__device__ __forceinline__ Item item_geometry(const AttnTile* __restrict__ tiles, int ntiles, int u, int window) {
  Item it;
  it.head = u / ntiles;
  it.tl = tiles[u % ntiles];
  int kend = it.tl.kv_len;
  it.kbeg = 0;
  if (window >= 0) {
    it.kbeg = max(0, it.tl.q_pos0 - window);
    kend = min(it.tl.kv_len, it.tl.q_pos0 + it.tl.nq + window);
  }
  it.nb = (kend - it.kbeg + KB - 1) / KB;
  return it;
}

__global__ void __launch_bounds__(192, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                   const __grid_constant__ CUtensorMap tmO, int use_tma_out, const AttnTile* __restrict__ tiles,
                   int ntiles, int heads, bf16* __restrict__ out, int ldo, int q_col0, int k_col0, int v_col0,
                   int window, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                 // 2 buffers
  uint8_t* sK = sQ + 2 * TILE_BYTES;  // 2 stages
  uint8_t* sV = sK + 2 * TILE_BYTES;  // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * TILE_BYTES);
  uint64_t* kv_full = bars + 0;  // [2] per stage
  uint64_t* kv_free = bars + 2;  // [2] per stage
  uint64_t* q_full = bars + 4;   // [2] per Q buffer
  uint64_t* q_free = bars + 6;   // [2] per Q buffer
  uint64_t* s_full = bars + 8;   // S of the next block in TMEM (and the P.V before the previous one)
  uint64_t* p_full = bars + 9;   // P of the current block in TMEM (one arrival per softmax warp)
  uint64_t* o_full = bars + 10;  // last P.V of an item done
  uint64_t* drain = bars + 11;
  uint64_t* pv_full = bars + 12;  // P.V of a block other than an item's last done (P may be rewritten)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int items = ntiles * heads;
  {  // exit before allocating anything when an earlier CTA of this launch gave up
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = device_aborted(err) ? 1 : 0;
    __syncthreads();
    if (s_abort) return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_free[i], 1);
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 4);  // one arrival per softmax warp (its rows of O have left)
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(pv_full, 1);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t kvb = 0;  // K/V blocks loaded so far (stage = kvb & 1)
      uint32_t armed_kv[2] = {0u, 0u}, armed_q[2] = {0u, 0u};  // parity+1 of the last armed phases
      int n = 0;         // items handled by this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < items && ok; u += gridDim.x, ++n) {
        const Item it = item_geometry(tiles, ntiles, u, window);
        const int qb = n & 1;
        // the Q buffer of item n - 2 is free once its O has left through it (softmax storer)
        if (n >= 2 && !mbar_wait(&q_free[qb], ((n - 2) >> 1) & 1, abort_flag, err, 10)) break;
        mbar_arrive_expect_tx(&q_full[qb], TILE_BYTES);
        tma_load_2d(&tmQ, &q_full[qb], sQ + qb * TILE_BYTES, q_col0 + it.head * HD, it.tl.q_row0);
        armed_q[qb] = 1 + ((n >> 1) & 1);
        for (int j = 0; j < it.nb; ++j, ++kvb) {
          const int st = kvb & 1;
          if (kvb >= 2 && !mbar_wait(&kv_free[st], ((kvb - 2) >> 1) & 1, abort_flag, err, 11)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * TILE_BYTES);
          const int krow = it.tl.kv_row0 + it.kbeg + j * KB;
          tma_load_2d(&tmKV, &kv_full[st], sK + st * TILE_BYTES, k_col0 + it.head * HD, krow);
          tma_load_2d(&tmKV, &kv_full[st], sV + st * TILE_BYTES, v_col0 + it.head * HD, krow);
          armed_kv[st] = 1 + ((kvb >> 1) & 1);
        }
      }
      if (*abort_flag) {  // let copies in flight land before smem is released
        volatile int no_abort = 0;
        for (int s = 0; s < 2; ++s) {
          if (armed_q[s]) mbar_wait(&q_full[s], armed_q[s] - 1, &no_abort, nullptr, 0);
          if (armed_kv[s]) mbar_wait(&kv_full[s], armed_kv[s] - 1, &no_abort, nullptr, 0);
        }
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    // Per block: wait for P(j); issue the next S (S(j+1), or S(0) of the next item) so that
    // the softmax can start on it at once; then P(j).V(j) into O.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = idesc_bf16(128, 64, false, true);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK), v0 = smem_u32(sV);
      uint32_t pcnt = 0;  // p_full phases consumed
      uint32_t kvb = 0;   // K/V blocks of earlier items
      bool ok = true;
      auto issue_s = [&](int n, uint32_t b) -> bool {  // S = Q(item n) K(block b)^T
        if (!mbar_wait(&kv_full[b & 1], (b >> 1) & 1, abort_flag, err, 13)) return false;
        tc_fence_after();
        const uint32_t qa = q0 + (n & 1) * TILE_BYTES, kb = k0 + (b & 1) * TILE_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem_base + TS_COL, sdesc_sw128(qa + k * 32, 16, 1024), sdesc_sw128(kb + k * 32, 16, 1024), idS,
                    k > 0);
        umma_commit(s_full);  // also covers every P.V issued before it
        return true;
      };
      auto wait_q = [&](int n) { return mbar_wait(&q_full[n & 1], (n >> 1) & 1, abort_flag, err, 12); };
      int n = 0;
      if (blockIdx.x < items) ok = wait_q(0) && issue_s(0, 0);
      for (int u = blockIdx.x; u < items && ok; u += gridDim.x, ++n) {
        const Item it = item_geometry(tiles, ntiles, u, window);
        const bool has_next = u + static_cast<int>(gridDim.x) < items;
        for (int j = 0; j < it.nb; ++j) {
          // P(j) is in TMEM and the group has finished reading S(j)
          if (!mbar_wait(p_full, pcnt & 1, abort_flag, err, 14)) {
            ok = false;
            break;
          }
          ++pcnt;
          tc_fence_after();
          const uint32_t b = kvb + j;
          if (j + 1 < it.nb) ok = issue_s(n, b + 1);
          else if (has_next) ok = wait_q(n + 1) && issue_s(n + 1, b + 1);
          if (!ok) break;
          const uint32_t vb0 = v0 + (b & 1) * TILE_BYTES;
#pragma unroll
          for (int k = 0; k < KB / 16; ++k)
            umma_bf16_ts(tmem_base + TO_COL, tmem_base + TP_COL + k * 8, sdesc_sw128(vb0 + k * 2048, 8192, 1024), idO,
                         (k > 0 || j > 0) ? 1u : 0u);
          umma_commit(&kv_free[b & 1]);
          // P(j) consumed: the softmax may write P(j+1); after the last block, O is final
          umma_commit(j + 1 < it.nb ? pv_full : o_full);
        }
        kvb += it.nb;
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int r = threadIdx.x;  // query row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem_base + TS_COL + lane_off, tP = tmem_base + TP_COL + lane_off;
    const uint32_t tO = tmem_base + TO_COL + lane_off;
    constexpr float kRescaleLog2 = 8.f;
    uint32_t ns = 0, no = 0, npv = 0;  // s_full / o_full / pv_full phases consumed
    bool ok = true;
    // The epilogue of an item (O / l -> ctx) runs while the next item's first block is in
    // progress: its O is complete once o_full fires, and it must be read before this
    // group's next p_full lets P.V(0) of the next item overwrite it.
    struct Pending {
      bool on;
      float l;
      int row0, nq, head, qb;
    } pend = {false, 0.f, 0, 0, 0, 0};
    auto epilogue = [&]() {
      const float inv = pend.l > 0.f ? 1.f / pend.l : 0.f;
      uint32_t orr[2][32];
      tmem_ld32(tO, orr[0]);
      tmem_ld32(tO + 32, orr[1]);
      tmem_ld_wait();
      uint4 w[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const uint32_t* v = &orr[g >> 2][(g & 3) * 8];
        w[g].x = pack_bf16x2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv);
        w[g].y = pack_bf16x2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv);
        w[g].z = pack_bf16x2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv);
        w[g].w = pack_bf16x2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv);
      }
      tc_fence_before();  // O read before the next p_full
      const int w0 = warp * 32;  // this warp's 32 rows of the tile
      if (use_tma_out && w0 + 32 <= pend.nq) {
        // stage the warp's 32 x 64 rows in the item's Q buffer (128B swizzle, the TMA
        // layout) and write them with one TMA store; lane 0 hands its part of the buffer
        // back to the producer once the store has read it
        uint8_t* row = sQ + pend.qb * TILE_BYTES + r * 128;
#pragma unroll
        for (int g = 0; g < 8; ++g)
          *reinterpret_cast<uint4*>(row + ((static_cast<uint32_t>(g) ^ (r & 7)) << 4)) = w[g];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (!*abort_flag) {
            tma_store_2d(&tmO, sQ + pend.qb * TILE_BYTES + w0 * 128, pend.head * HD, pend.row0 + w0);
            bulk_commit();
            bulk_wait_read_all();
          }
          mbar_arrive(&q_free[pend.qb]);
        }
      } else {  // rows past the tile's end (ragged tail) or no output map: plain stores
        if (r < pend.nq) {
          uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(pend.row0 + r) * ldo + pend.head * HD);
#pragma unroll
          for (int g = 0; g < 8; ++g) dst[g] = w[g];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_free[pend.qb]);
      }
      pend.on = false;
    };
    int n = 0;
    for (int u = blockIdx.x; u < items && ok; u += gridDim.x, ++n) {
      const Item it = item_geometry(tiles, ntiles, u, window);
      const int qpos = it.tl.q_pos0 + r;
      // this row's valid keys: [klo, khi)
      const int klo = window >= 0 ? max(0, qpos - window) : 0;
      const int khi = window >= 0 ? min(it.tl.kv_len, qpos + window + 1) : it.tl.kv_len;
      float m_used = -INFINITY;  // offset of P and O (scaled, base 2)
      float l = 0.f;
      for (int j = 0; j < it.nb; ++j, ++ns) {
        if (!warp_wait(s_full, ns & 1, abort_flag, err, 16)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int key0 = it.kbeg + j * KB;
        // valid columns c of this block: lo <= c < hi, tested as (unsigned)(c - lo) < span.
        // Masked scores become -inf *before* the exponential (a select around ex2 would
        // cost ~3x in issue slots).
        const int lo = klo - key0;
        const unsigned span = static_cast<unsigned>(max(khi - klo, 0));
        if (j == 0) {
          // first block: exact row max before the exponentials
          float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
          for (int c = 0; c < KB / 32; ++c) {
            uint32_t sr[32];
            tmem_ld32(tS + c * 32, sr);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const bool v = static_cast<unsigned>(c * 32 + i - lo) < span;
              mxp[i & 3] = fmaxf(mxp[i & 3], v ? __uint_as_float(sr[i]) : -INFINITY);
            }
          }
          m_used = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])) * scale_log2;
        }
        // exponentiate with the current offset; redo once if the block max moved it too far
        float lb = 0.f;
        // before P is written: the previous P.V must have read P (and finished adding to O)
        bool p_wait = j > 0 || pend.on;
        for (int attempt = 0; attempt < 2; ++attempt) {
          const float uu = (m_used == -INFINITY) ? 0.f : m_used;
          float lp[4] = {0.f, 0.f, 0.f, 0.f};
          float bm[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
          for (int c = 0; c < KB / 64; ++c) {
            uint32_t sa[32], sb[32];
            tmem_ld32(tS + c * 64, sa);
            tmem_ld32(tS + c * 64 + 32, sb);
            tmem_ld_wait();
            uint32_t pk[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = c * 64 + 2 * i;
              const float s0 = __uint_as_float(i < 16 ? sa[2 * i] : sb[2 * i - 32]);
              const float s1 = __uint_as_float(i < 16 ? sa[2 * i + 1] : sb[2 * i - 31]);
              const float a0 = static_cast<unsigned>(col - lo) < span ? s0 : -INFINITY;
              const float a1 = static_cast<unsigned>(col + 1 - lo) < span ? s1 : -INFINITY;
              const float p0 = ex2(fmaf(a0, scale_log2, -uu));
              const float p1 = ex2(fmaf(a1, scale_log2, -uu));
              bm[i & 3] = fmaxf(bm[i & 3], a0);
              bm[(i + 2) & 3] = fmaxf(bm[(i + 2) & 3], a1);
              lp[i & 3] += p0 + p1;
              pk[i] = pack_bf16x2(p0, p1);
            }
            if (p_wait) {
              const bool w = j > 0 ? warp_wait(pv_full, npv & 1, abort_flag, err, 15)
                                   : warp_wait(o_full, no & 1, abort_flag, err, 18);
              if (j > 0) ++npv;
              else ++no;
              if (!w) ok = false;
              p_wait = false;
              tc_fence_after();
            }
            tmem_st32(tP + c * 32, pk);
          }
          tmem_st_wait();
          lb = (lp[0] + lp[1]) + (lp[2] + lp[3]);
          const float bmax = fmaxf(fmaxf(bm[0], bm[1]), fmaxf(bm[2], bm[3])) * scale_log2;
          const bool moved = bmax > m_used + kRescaleLog2;  // never on the first block
          if (!__any_sync(0xffffffffu, moved)) break;
          // some row of this warp needs a larger offset: rescale its O and l, redo the block
          const float m_new = moved ? bmax : m_used;
          const float alpha = moved ? ex2(m_used - m_new) : 1.f;
          l *= alpha;
          m_used = m_new;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            uint32_t orr[32];
            tmem_ld32(tO + h * 32, orr);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) orr[i] = __float_as_uint(__uint_as_float(orr[i]) * alpha);
            tmem_st32(tO + h * 32, orr);
          }
          tmem_st_wait();
        }
        if (!ok) break;
        l += lb;
        if (pend.on) epilogue();  // previous item's O (complete: o_full was waited above)
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      pend = {true, l, it.tl.q_row0, it.tl.nq, it.head, n & 1};
    }
    if (ok && pend.on) {
      if (warp_wait(o_full, no & 1, abort_flag, err, 18)) {
        ++no;
        tc_fence_after();
        epilogue();
      }
    }
    if (lane == 0) bulk_wait_all();  // no store of ours may still read smem at exit
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem_base, 256);
}

}  // namespace

int attention_pair_queries() { return QT; }

int launch_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, const CUtensorMap* tmO, const AttnTile* tiles,
                     int ntiles, int heads, int q_col0, int k_col0, int v_col0, bf16* out, int ldo, int window,
                     float scale_log2, int* err, int grid_limit, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};  // one bit per device
  const cudaError_t e = set_smem_once(attn_tc_kernel, ATT_SMEM, configured);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (ntiles == 0 || heads == 0) return 0;
  const int items = ntiles * heads;
  const int limit = 2 * grid_limit;  // two CTAs per SM
  const int grid = items < limit ? items : limit;
  attn_tc_kernel<<<grid, 192, ATT_SMEM, stream>>>(tmQ, tmKV, tmO ? *tmO : tmQ, tmO ? 1 : 0, tiles, ntiles, heads,
                                                   out, ldo, q_col0, k_col0, v_col0, window, scale_log2, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace j1rt
