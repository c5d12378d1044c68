// Varlen FlashAttention-style kernel on tcgen05 / TMEM for head_dim 64.
//
// Replaces the reference's mma.sync kernel `attention_impl` (src/cuda/kernels.cu:272-391)
// with the same semantics: packed sequences without padding, online softmax in base 2
// with scale 0.125*log2(e), an optional |i - j| <= window band (local layers,
// kernels.cu:304-308,332), and P rounded to BF16 before P.V. RoPE is not applied here:
// the Wqkv GEMM epilogue already rotated q and k.
//
// Work item = two consecutive 128-query tiles of one sequence x one head (a "tile pair").
// The kernel is persistent: one CTA per SM walks items blockIdx.x, +gridDim.x, ... with
// barrier phases, TMEM and smem set up once; Q is double buffered so the producer
// fetches the next item's Q and K/V while the current item computes. 320 threads:
//   warps 0..3  softmax of tile 0, warps 4..7 softmax of tile 1: thread r of a group owns
//               query row r (TMEM lane r); reads S from TMEM, writes P (bf16, 128B-swizzled,
//               K-major) to smem; O accumulates in TMEM across the item's key blocks
//   warp 8      tcgen05.mma issuer: S_t = Q_t K^T (M=128, N=128, K=64) and
//               O_t = P_t V (M=128, N=64, K=128; V read MN-major)
//   warp 9      TMA producer: Q_0/Q_1 per item, K/V blocks of 128 keys, double buffered
// The two tiles share every K/V block they both need; the issuer runs the P.V of one
// tile and the next Q.K^T of that tile while the other tile's softmax is in flight.
// TMEM (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256,320), O_1 [320,384).
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
constexpr uint32_t P_BYTES = QT * KB * 2;      // 32 KB
constexpr uint32_t ATT_SMEM = 8 * TILE_BYTES + 2 * P_BYTES + 1024 + 256;

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

// Geometry of one work item (identical in every role of the CTA).
struct Item {
  AttnTile tl;
  int head, kbeg, nb;
  int jb0, je0, jb1, je1, nq0, nq1;
};

__device__ __forceinline__ Item item_geometry(const AttnTile* __restrict__ tiles, int npairs, int u, int window) {
  Item it;
  it.head = u / npairs;
  it.tl = tiles[u % npairs];
  const AttnTile& tl = it.tl;
  int kend = tl.kv_len;
  it.kbeg = 0;
  if (window >= 0) {
    it.kbeg = max(0, tl.q_pos0 - window);
    kend = min(tl.kv_len, tl.q_pos0 + tl.nq + window);
  }
  it.nb = (kend - it.kbeg + KB - 1) / KB;
  int jb[2], je[2], nq[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    nq[t] = min(max(tl.nq - QT * t, 0), QT);
    const int qp = tl.q_pos0 + QT * t;
    if (nq[t] == 0) {
      jb[t] = je[t] = 0;
    } else if (window < 0) {
      jb[t] = 0;
      je[t] = it.nb;
    } else {
      const int lo = max(0, qp - window), hi = min(tl.kv_len, qp + nq[t] + window);
      jb[t] = (lo - it.kbeg) / KB;
      je[t] = (hi - it.kbeg + KB - 1) / KB;
    }
  }
  it.jb0 = jb[0], it.je0 = je[0], it.jb1 = jb[1], it.je1 = je[1], it.nq0 = nq[0], it.nq1 = nq[1];
  return it;
}

__global__ void __launch_bounds__(320, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                   const AttnTile* __restrict__ tiles, int npairs, int heads, bf16* __restrict__ out, int ldo,
                   int q_col0, int k_col0, int v_col0, int window, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                     // 2 buffers x 2 tiles
  uint8_t* sK = sQ + 4 * TILE_BYTES;      // 2 stages
  uint8_t* sV = sK + 2 * TILE_BYTES;      // 2 stages
  uint8_t* sP = sV + 2 * TILE_BYTES;      // 2 tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_BYTES);
  uint64_t* kv_full = bars + 0;   // [2] per stage
  uint64_t* kv_free = bars + 2;   // [2] per stage
  uint64_t* s_full = bars + 4;    // [2] per tile
  uint64_t* p_full = bars + 6;    // [2] per tile
  uint64_t* o_full = bars + 8;    // [2] per tile
  uint64_t* q_full = bars + 10;   // [2] per Q buffer
  uint64_t* q_free = bars + 12;   // [2] per Q buffer
  uint64_t* drain = bars + 14;
  uint64_t* s_free = bars + 16;   // [2] per tile: the group has read S_t into registers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const int items = npairs * heads;
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
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 1);
      mbar_init(&s_free[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t kvb = 0;                           // K/V blocks loaded so far (stage = kvb & 1)
      uint32_t armed_kv[2] = {0u, 0u}, armed_q[2] = {0u, 0u};  // parity+1 of the last armed phases
      int n = 0;                                  // items handled by this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < items && ok; u += gridDim.x, ++n) {
        const Item it = item_geometry(tiles, npairs, u, window);
        const int qb = n & 1;
        if (n >= 2 && !mbar_wait(&q_free[qb], ((n - 2) >> 1) & 1, abort_flag, err, 10)) break;
        mbar_arrive_expect_tx(&q_full[qb], it.nq1 > 0 ? 2 * TILE_BYTES : TILE_BYTES);
        uint8_t* qdst = sQ + qb * 2 * TILE_BYTES;
        tma_load_2d(&tmQ, &q_full[qb], qdst, q_col0 + it.head * HD, it.tl.q_row0);
        if (it.nq1 > 0) tma_load_2d(&tmQ, &q_full[qb], qdst + TILE_BYTES, q_col0 + it.head * HD, it.tl.q_row0 + QT);
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
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = idesc_bf16(128, 64, false, true);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK), v0 = smem_u32(sV), p0 = smem_u32(sP);
      uint32_t pcnt0 = 0, pcnt1 = 0;  // p_full phases consumed per tile
      uint32_t scnt[2] = {0u, 0u};    // S MMAs issued per tile (s_free phases trail by one)
      uint32_t kvb = 0;               // K/V blocks consumed so far
      int n = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < items && ok; u += gridDim.x, ++n) {
        const Item it = item_geometry(tiles, npairs, u, window);
        const int qb = n & 1;
        if (!mbar_wait(&q_full[qb], (n >> 1) & 1, abort_flag, err, 12)) break;
        const uint32_t qbase = q0 + qb * 2 * TILE_BYTES;
        auto issue_s = [&](int t, int j) -> bool {
          // S_t is overwritten: the group must have read the previous S_t into registers
          if (scnt[t] > 0 && !mbar_wait(&s_free[t], (scnt[t] - 1) & 1, abort_flag, err, 19)) return false;
          ++scnt[t];
          const uint32_t b = kvb + j;  // global block index of item block j
          if (!mbar_wait(&kv_full[b & 1], (b >> 1) & 1, abort_flag, err, 13)) return false;
          tc_fence_after();
          const uint32_t qa = qbase + t * TILE_BYTES, kb = k0 + (b & 1) * TILE_BYTES;
#pragma unroll
          for (int k = 0; k < HD / 16; ++k)
            umma_bf16(tmem_base + t * 128, sdesc_sw128(qa + k * 32, 16, 1024), sdesc_sw128(kb + k * 32, 16, 1024),
                      idS, k > 0);
          umma_commit(&s_full[t]);
          return true;
        };
        auto issue_pv = [&](int t, int j, uint32_t& pcnt, bool first) -> bool {
          // P_t(j) is in smem (and O_t rescaled by the group when its offset moved)
          if (!mbar_wait(&p_full[t], pcnt & 1, abort_flag, err, 14)) return false;
          ++pcnt;
          tc_fence_after();
          const uint32_t b = kvb + j;
          const uint32_t pa0 = p0 + t * P_BYTES, vb0 = v0 + (b & 1) * TILE_BYTES;
#pragma unroll
          for (int k = 0; k < KB / 16; ++k) {
            const uint32_t pa = pa0 + (k >> 2) * (QT * 128) + (k & 3) * 32;
            umma_bf16(tmem_base + 256 + t * 64, sdesc_sw128(pa, 16, 1024), sdesc_sw128(vb0 + k * 2048, 8192, 1024),
                      idO, (k > 0 || !first) ? 1u : 0u);  // O_t accumulates over the item's blocks
          }
          umma_commit(&o_full[t]);
          return true;
        };
        for (int j = 0; j < it.nb && ok; ++j) {
          const bool a0 = j >= it.jb0 && j < it.je0, a1 = j >= it.jb1 && j < it.je1;
          if (j == it.jb0 && a0) ok = issue_s(0, j);
          if (ok && j == it.jb1 && a1) ok = issue_s(1, j);
          // next Q.K^T of each tile as soon as its group has pulled S into registers ...
          if (ok && a0 && j + 1 < it.je0) ok = issue_s(0, j + 1);
          if (ok && a1 && j + 1 < it.je1) ok = issue_s(1, j + 1);
          // ... then P.V once the group has written P
          if (ok && a0) ok = issue_pv(0, j, pcnt0, j == it.jb0);
          if (ok && a1) ok = issue_pv(1, j, pcnt1, j == it.jb1);
          umma_commit(&kv_free[(kvb + j) & 1]);
        }
        umma_commit(&q_free[qb]);  // every S of this item read Q[qb]
        kvb += it.nb;
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warps (group t)
    // S is read from TMEM once per block (128 columns -> registers). O stays in TMEM and is
    // accumulated by the P.V MMAs; P and O share an offset u (base-2, scaled) that only
    // moves when the running max exceeds it by more than 2^8, in which case the group
    // rescales O in TMEM before releasing the next P. P <= 2^8 then, and BF16 rounding of
    // P is relative, so the result matches always-rescaled online softmax to rounding.
    const int t = warp >> 2;
    const int r = threadIdx.x & 127;  // query row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + t * 128 + lane_off, tO = tmem_base + 256 + t * 64 + lane_off;
    uint8_t* prow = sP + t * P_BYTES + r * 128;
    const uint32_t sw = static_cast<uint32_t>(r & 7);
    constexpr float kRescaleLog2 = 8.f;
    uint32_t ns = 0;  // S / O phases consumed by this group
    bool ok = true;
    for (int u = blockIdx.x; u < items && ok; u += gridDim.x) {
      const Item it = item_geometry(tiles, npairs, u, window);
      const int jb = t ? it.jb1 : it.jb0, je = t ? it.je1 : it.je0, nq = t ? it.nq1 : it.nq0;
      if (jb >= je) continue;  // this tile of the pair is empty
      const int qpos = it.tl.q_pos0 + QT * t + r;
      // this row's valid keys: [klo, khi)
      const int klo = window >= 0 ? max(0, qpos - window) : 0;
      const int khi = window >= 0 ? min(it.tl.kv_len, qpos + window + 1) : it.tl.kv_len;
      float m_used = -INFINITY;  // offset of P and O (scaled, base 2)
      float l = 0.f;
      for (int j = jb; j < je; ++j, ++ns) {
        if (!warp_wait(&s_full[t], ns & 1, abort_flag, err, 16)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[KB / 32][32];
#pragma unroll
        for (int c = 0; c < KB / 32; ++c) tmem_ld32(tS + c * 32, sr[c]);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&s_free[t]);  // S_t may be overwritten by the next Q.K^T
        const int key0 = it.kbeg + j * KB;
        const int lo = klo - key0, hi = khi - key0;  // valid columns c: lo <= c < hi
        const bool all_valid = lo <= 0 && hi >= KB;
        float mxp[8];  // independent partial maxima (short dependency chains)
#pragma unroll
        for (int k = 0; k < 8; ++k) mxp[k] = -INFINITY;
#pragma unroll
        for (int c = 0; c < KB / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = c * 32 + i;
            const float v = __uint_as_float(sr[c][i]);
            mxp[i & 7] = (all_valid || (col >= lo && col < hi)) ? fmaxf(mxp[i & 7], v) : mxp[i & 7];
          }
        const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                               fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        const float m_cand = fmaxf(m_used, mx * scale_log2);
        float alpha = 1.f;
        bool moved = false;
        if (m_cand > m_used + kRescaleLog2) {
          alpha = ex2(m_used - m_cand);
          l *= alpha;
          m_used = m_cand;
          moved = true;
        }
        const float uu = (m_used == -INFINITY) ? 0.f : m_used;
        // P_t(j) replaces P_t(j-1): the P.V of the previous block must be complete
        if (j > jb) {
          if (!warp_wait(&o_full[t], (ns - 1) & 1, abort_flag, err, 17)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        // P = 2^(s*scale - u) as bf16 into the swizzled K-major P tile
        float lp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // partial row sums
#pragma unroll
        for (int c = 0; c < KB / 32; ++c) {
          float pv[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = c * 32 + i;
            const float e = ex2(fmaf(__uint_as_float(sr[c][i]), scale_log2, -uu));
            pv[i] = (all_valid || (col >= lo && col < hi)) ? e : 0.f;
            lp[i & 7] += pv[i];
          }
          // keys c*32 .. c*32+31 live in K-chunk c/2 (64 keys), 16-byte units (c&1)*4 .. +3
          uint8_t* chunk = prow + (c >> 1) * (QT * 128);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const uint32_t unit = static_cast<uint32_t>((c & 1) * 4 + g);
            uint4 w;
            w.x = pack_bf16x2(pv[8 * g + 0], pv[8 * g + 1]);
            w.y = pack_bf16x2(pv[8 * g + 2], pv[8 * g + 3]);
            w.z = pack_bf16x2(pv[8 * g + 4], pv[8 * g + 5]);
            w.w = pack_bf16x2(pv[8 * g + 6], pv[8 * g + 7]);
            *reinterpret_cast<uint4*>(chunk + ((unit ^ sw) << 4)) = w;
          }
        }
        l += ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
        // O_t(j-1) is complete (waited above): move it to the new offset before P_t(j).V accumulates.
        // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp takes this branch
        // when any of its rows moved; rows that did not move scale by 1.
        if (j > jb && __any_sync(0xffffffffu, moved)) {
          if (!moved) alpha = 1.f;
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
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
      if (!ok || !warp_wait(&o_full[t], (ns - 1) & 1, abort_flag, err, 18)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint32_t orr[2][32];
      tmem_ld32(tO, orr[0]);
      tmem_ld32(tO + 32, orr[1]);
      tmem_ld_wait();
      if (r < nq) {
        uint4* dst =
            reinterpret_cast<uint4*>(out + static_cast<size_t>(it.tl.q_row0 + QT * t + r) * ldo + it.head * HD);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const uint32_t* v = &orr[g >> 2][(g & 3) * 8];
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv);
          dst[g] = w;
        }
      }
      // O_t is reused by the next item's first P.V (issued after this group's next p_full)
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) tmem_dealloc(tmem_base, 512);
}

}  // namespace

int attention_pair_queries() { return 2 * QT; }

int launch_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, const AttnTile* tiles, int ntiles, int heads,
                     int q_col0, int k_col0, int v_col0, bf16* out, int ldo, int window, float scale_log2, int* err,
                     int grid_limit, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
  if (ntiles == 0 || heads == 0) return 0;
  const int items = ntiles * heads;
  const int grid = items < grid_limit ? items : grid_limit;
  attn_tc_kernel<<<grid, 320, ATT_SMEM, stream>>>(tmQ, tmKV, tiles, ntiles, heads, out, ldo, q_col0, k_col0, v_col0,
                                                   window, scale_log2, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace j1rt
