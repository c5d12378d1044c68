// Varlen FlashAttention-style kernel on tcgen05 / TMEM for head_dim 64.
//
// Replaces the reference's mma.sync kernel `attention_impl` (src/cuda/kernels.cu:272-391)
// with the same semantics: packed sequences without padding, online softmax in base 2
// with scale 0.125*log2(e), an optional |i - j| <= window band (local layers,
// kernels.cu:304-308,332), and P rounded to BF16 before P.V. RoPE is not applied here:
// the Wqkv GEMM epilogue already rotated q and k.
//
// Work item = one 128-query tile of one sequence x one head; its keys are visited in
// blocks of 64. The kernel is persistent with two CTAs per SM (one CTA's softmax
// overlaps the other's); each CTA walks items blockIdx.x, +gridDim.x, ... and treats
// the key blocks of all its items as one stream g = 0, 1, 2, ... 192 threads per CTA:
//   warps 0..3  softmax: thread r owns query row r (TMEM lane r); reads S(g) from TMEM
//               into registers, writes P(g) (bf16 pairs) back to TMEM; O accumulates
//               in TMEM over an item's blocks
//   warp 4      tcgen05.mma issuer: S = Q K^T (M=128, N=64, K=64, operands in smem) and
//               O += P V (M=128, N=64, K=64; P from TMEM, V from smem read MN-major)
//   warp 5      TMA producer: Q (double buffered across items), K/V blocks (4 stages)
// TMEM (256 columns): S(g) in [64 (g&1), +64); P(g) overwrites the first 32 of those
// columns once the row's scores are in registers; O of the CTA's n-th item in
// [128 + 64 (n&1), +64). With S double buffered the MMA runs two blocks ahead of the
// softmax: S(g+2) is issued once P(g).V(g) has read P(g), so the softmax rarely waits
// for S. With O double buffered the next item's P.V never waits for an epilogue.
//
// Softmax per block: the 64 scores of the row are loaded once and their exact maximum
// is taken first; the running offset only moves (rescaling O and l) when the maximum
// grew by more than 2^8, so P <= 2^8 and BF16 rounding of P stays relative: the result
// matches the always-rescaled online softmax to rounding. Blocks that are fully masked
// for all 32 rows of a warp skip the exponentials (P = 0).
//
// The epilogue of an item (O / l -> out) runs during the first block of the next item,
// after that block's P is handed over; full 32-row slices leave by TMA store, staged in
// the item's Q buffer, which goes back to the producer one block later (once the store
// has read it), or before the next S wait when that S needs the buffer's next Q.
#include <cuda.h>
#include <cuda_runtime.h>

#include "kernels.h"
#include "ptx.cuh"

namespace j1rt {

namespace {

constexpr int QT = 128;  // queries per tile
constexpr int KB = 64;   // keys per block
constexpr int HD = 64;   // head dim
constexpr int NKV = 4;   // K/V stages
constexpr uint32_t Q_BYTES = QT * HD * 2;   // 16 KB Q box
constexpr uint32_t KV_BYTES = KB * HD * 2;  // 8 KB K or V box
constexpr uint32_t ATT_SMEM = 2 * Q_BYTES + NKV * 2 * KV_BYTES + 1024 + 256;
constexpr uint32_t TS_COL = 0, TO_COL = 128;

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

__device__ __forceinline__ Item item_geometry(const AttnTile& tl, int ntiles, int u, int window) {
  Item it;
  it.head = u / ntiles;
  it.tl = tl;
  int kend = it.tl.kv_len;
  it.kbeg = 0;
  if (window >= 0) {
    it.kbeg = max(0, it.tl.q_pos0 - window);
    kend = min(it.tl.kv_len, it.tl.q_pos0 + it.tl.nq + window);
  }
  it.nb = (kend - it.kbeg + KB - 1) / KB;
  return it;
}

__device__ __forceinline__ AttnTile load_tile(const AttnTile* __restrict__ tiles, int ntiles, int u, int items) {
  AttnTile t = {0, 0, 0, 0, 0, 0, 0, 0};
  if (u < items) t = tiles[u % ntiles];
  return t;
}

// Walks the (item, block) stream of one CTA: item u (the n-th of this CTA), block j.
// The tile record of the following item is fetched one item ahead.
struct Cursor {
  int u, n, j;
  Item it;
  AttnTile next;
};
__device__ __forceinline__ void cursor_start(Cursor& c, const AttnTile* tiles, int ntiles, int items, int window) {
  c.u = blockIdx.x;
  c.n = 0;
  c.j = 0;
  if (c.u < items) c.it = item_geometry(tiles[c.u % ntiles], ntiles, c.u, window);
  c.next = load_tile(tiles, ntiles, c.u + static_cast<int>(gridDim.x), items);
}
__device__ __forceinline__ void cursor_next(Cursor& c, const AttnTile* tiles, int ntiles, int items, int window) {
  if (++c.j < c.it.nb) return;
  c.j = 0;
  c.u += gridDim.x;
  ++c.n;
  if (c.u < items) {
    c.it = item_geometry(c.next, ntiles, c.u, window);
    c.next = load_tile(tiles, ntiles, c.u + static_cast<int>(gridDim.x), items);
  }
}

__global__ void __launch_bounds__(192, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                   const __grid_constant__ CUtensorMap tmO, int use_tma_out, const AttnTile* __restrict__ tiles,
                   int ntiles, int heads, bf16* __restrict__ out, int ldo, int q_col0, int k_col0, int v_col0,
                   int window, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                 // 2 buffers
  uint8_t* sK = sQ + 2 * Q_BYTES;     // NKV stages
  uint8_t* sV = sK + NKV * KV_BYTES;  // NKV stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NKV * KV_BYTES);
  uint64_t* kv_full = bars;           // [NKV]
  uint64_t* pv_done = bars + NKV;     // [NKV] per K/V stage: P(g).V(g) done (stage g % NKV free)
  uint64_t* q_full = bars + 2 * NKV;  // [2] per Q buffer
  uint64_t* q_free = q_full + 2;      // [2] per Q buffer (one arrival per softmax warp)
  uint64_t* s_full = q_free + 2;      // [2] per S buffer: S(g) in TMEM
  uint64_t* p_full = s_full + 2;      // [2] per S buffer: P(g) written over S(g) (4 arrivals)
  uint64_t* o_full = p_full + 2;      // [2] per O buffer: last P.V of an item done
  uint64_t* drain = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  grid_dep_launch();
  const int warp = warp_id(), lane = lane_id();
  const int items = ntiles * heads;
  {  // exit before allocating anything when an earlier CTA of this launch gave up
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = device_aborted(err) ? 1 : 0;
    __syncthreads();
    if (s_abort) return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < NKV; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&pv_done[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_free[i], 4);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
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
  grid_dep_wait();  // the previous kernel's outputs (this kernel's inputs and outputs) are ready
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t g = 0;  // K/V blocks loaded so far (stage = g % NKV)
      uint32_t armed_kv[NKV] = {0u, 0u, 0u, 0u}, armed_q[2] = {0u, 0u};  // parity+1 of the last armed phases
      int n = 0;       // items handled by this CTA
      bool ok = true;
      for (int u = blockIdx.x; u < items && ok; u += gridDim.x, ++n) {
        const Item it = item_geometry(tiles[u % ntiles], ntiles, u, window);
        const int qb = n & 1;
        // the Q buffer of item n - 2 is free once its O has left through it (softmax)
        if (n >= 2 && !mbar_wait(&q_free[qb], ((n - 2) >> 1) & 1, abort_flag, err, 10)) break;
        mbar_arrive_expect_tx(&q_full[qb], Q_BYTES);
        tma_load_2d(&tmQ, &q_full[qb], sQ + qb * Q_BYTES, q_col0 + it.head * HD, it.tl.q_row0);
        armed_q[qb] = 1 + ((n >> 1) & 1);
        for (int j = 0; j < it.nb; ++j, ++g) {
          const uint32_t st = g % NKV;
          if (g >= NKV && !mbar_wait(&pv_done[st], ((g - NKV) / NKV) & 1, abort_flag, err, 11)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * KV_BYTES);
          const int krow = it.tl.kv_row0 + it.kbeg + j * KB;
          tma_load_2d(&tmKV, &kv_full[st], sK + st * KV_BYTES, k_col0 + it.head * HD, krow);
          tma_load_2d(&tmKV, &kv_full[st], sV + st * KV_BYTES, v_col0 + it.head * HD, krow);
          armed_kv[st] = 1 + ((g / NKV) & 1);
        }
      }
      if (*abort_flag) {  // let copies in flight land before smem is released
        volatile int no_abort = 0;
        for (int s = 0; s < 2; ++s)
          if (armed_q[s]) mbar_wait(&q_full[s], armed_q[s] - 1, &no_abort, nullptr, 0);
        for (int s = 0; s < NKV; ++s)
          if (armed_kv[s]) mbar_wait(&kv_full[s], armed_kv[s] - 1, &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    // Block stream g: S(g) goes to S buffer g&1 once P(g-2) is in (the softmax has read
    // S(g-2)); P(g).V(g) follows P(g). So S runs two blocks ahead of P.V.
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, KB, false, false);
      constexpr uint32_t idO = idesc_bf16(128, HD, false, true);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK), v0 = smem_u32(sV);
      bool ok = true;
      int q_ready = -1;  // last item whose Q has been waited for
      // S(gs) for the block at cursor cs (item cs.n reads Q buffer cs.n & 1)
      auto issue_s = [&](const Cursor& cs, uint32_t gs) -> bool {
        if (cs.n > q_ready) {
          if (!mbar_wait(&q_full[cs.n & 1], (cs.n >> 1) & 1, abort_flag, err, 12)) return false;
          q_ready = cs.n;
        }
        const uint32_t st = gs % NKV;
        if (!mbar_wait(&kv_full[st], (gs / NKV) & 1, abort_flag, err, 13)) return false;
        tc_fence_after();
        const uint32_t qa = q0 + (cs.n & 1) * Q_BYTES, kb = k0 + st * KV_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem_base + TS_COL + (gs & 1) * KB, sdesc_sw128(qa + k * 32, 16, 1024),
                    sdesc_sw128(kb + k * 32, 16, 1024), idS, k > 0);
        umma_commit(&s_full[gs & 1]);
        return true;
      };
      Cursor cp, cs;  // P.V cursor (block g) and S cursor (block gs = g + 2)
      cursor_start(cp, tiles, ntiles, items, window);
      cursor_start(cs, tiles, ntiles, items, window);
      uint32_t gs = 0;
      for (; gs < 2 && cs.u < items && ok; ++gs) {
        ok = issue_s(cs, gs);
        cursor_next(cs, tiles, ntiles, items, window);
      }
      for (uint32_t g = 0; cp.u < items && ok; ++g) {
        // P(g) is in TMEM and the group has finished reading S(g)
        if (!mbar_wait(&p_full[g & 1], (g >> 1) & 1, abort_flag, err, 14)) break;
        tc_fence_after();
        const uint32_t vb0 = v0 + (g % NKV) * KV_BYTES;
        const uint32_t ob = static_cast<uint32_t>(cp.n & 1);
#pragma unroll
        for (int k = 0; k < KB / 16; ++k)
          umma_bf16_ts(tmem_base + TO_COL + ob * HD, tmem_base + TS_COL + (g & 1) * KB + k * 8,
                       sdesc_sw128(vb0 + k * 2048, 8192, 1024), idO, (k > 0 || cp.j > 0) ? 1u : 0u);
        umma_commit(&pv_done[g % NKV]);  // frees K/V stage g % NKV and S buffer g & 1
        if (cp.j + 1 == cp.it.nb) umma_commit(&o_full[ob]);  // O of the item is final
        cursor_next(cp, tiles, ntiles, items, window);
        if (cs.u < items) {
          // S(g+2) goes into the columns that hold P(g): P(g).V(g) must have read them
          if (!mbar_wait(&pv_done[g % NKV], (g / NKV) & 1, abort_flag, err, 19)) break;
          tc_fence_after();
          ok = issue_s(cs, gs);
          cursor_next(cs, tiles, ntiles, items, window);
          ++gs;
        }
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int r = threadIdx.x;  // query row == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    constexpr float kRescaleLog2 = 8.f;
    bool ok = true;
    // The epilogue of an item (O / l -> out) runs during the first block of the next
    // item, after that block's P is handed over: the next item accumulates into the
    // other O buffer, and o_full of this one has fired by then.
    struct Pending {
      bool on;
      float l;
      int row0, nq, head, n;  // n: the item's index in this CTA (O and Q buffer n & 1)
    } pend = {false, 0.f, 0, 0, 0, 0};
    int qrel = -1;  // Q buffer that a TMA store of ours may still be reading (warp-uniform)
    // Lane 0 hands the buffer back to the producer once the store has read it.
    auto release_q = [&]() {
      if (qrel >= 0) {
        if (lane == 0) {
          bulk_wait_read_all();
          mbar_arrive(&q_free[qrel]);
        }
        qrel = -1;
      }
    };
    auto epilogue = [&]() {
      const int ob = pend.n & 1;
      const uint32_t tO = tmem_base + TO_COL + ob * HD + lane_off;
      const float inv = pend.l > 0.f ? 1.f / pend.l : 0.f;
      uint32_t orr[2][32];
      tmem_ld32(tO, orr[0]);
      tmem_ld32(tO + 32, orr[1]);
      tmem_ld_wait();
      uint4 w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t* v = &orr[q >> 2][(q & 3) * 8];
        w[q].x = pack_bf16x2(__uint_as_float(v[0]) * inv, __uint_as_float(v[1]) * inv);
        w[q].y = pack_bf16x2(__uint_as_float(v[2]) * inv, __uint_as_float(v[3]) * inv);
        w[q].z = pack_bf16x2(__uint_as_float(v[4]) * inv, __uint_as_float(v[5]) * inv);
        w[q].w = pack_bf16x2(__uint_as_float(v[6]) * inv, __uint_as_float(v[7]) * inv);
      }
      tc_fence_before();  // O read before the next p_full
      const int w0 = warp * 32;  // this warp's 32 rows of the tile
      if (use_tma_out && w0 + 32 <= pend.nq) {
        // stage the warp's 32 x 64 rows in the item's Q buffer (128B swizzle, the TMA
        // layout) and write them with one TMA store; the buffer goes back to the producer
        // one block later (release_q)
        uint8_t* row = sQ + ob * Q_BYTES + r * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<uint4*>(row + ((static_cast<uint32_t>(q) ^ (r & 7)) << 4)) = w[q];
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && !*abort_flag) {
          tma_store_2d(&tmO, sQ + ob * Q_BYTES + w0 * 128, pend.head * HD, pend.row0 + w0);
          bulk_commit();
        }
        qrel = ob;
      } else {  // rows past the tile's end (ragged tail) or no output map: plain stores
        if (r < pend.nq) {
          uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(pend.row0 + r) * ldo + pend.head * HD);
#pragma unroll
          for (int q = 0; q < 8; ++q) dst[q] = w[q];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_free[ob]);
      }
      pend.on = false;
    };
    Cursor c;
    cursor_start(c, tiles, ntiles, items, window);
    float m_used = -INFINITY;  // offset of P and O (scaled, base 2)
    float l = 0.f;
    int klo = 0, khi = 0;  // this row's valid keys [klo, khi) within the current item
    for (uint32_t g = 0; c.u < items && ok; ++g) {
      const Item& it = c.it;
      if (c.j == 0) {
        release_q();  // this item's S may need the Q buffer of that store (the item after next)
        const int qpos = it.tl.q_pos0 + r;
        klo = window >= 0 ? max(0, qpos - window) : 0;
        khi = window >= 0 ? min(it.tl.kv_len, qpos + window + 1) : it.tl.kv_len;
        m_used = -INFINITY;
        l = 0.f;
      }
      const int key0 = it.kbeg + c.j * KB;
      // this block's valid columns for the row: [lo, lo + span), span possibly 0
      const int lo = max(klo - key0, 0), hi = min(khi - key0, KB);
      const unsigned span = static_cast<unsigned>(max(hi - lo, 0));
      const bool any = __any_sync(0xffffffffu, span > 0);
      const bool full = __all_sync(0xffffffffu, span == static_cast<unsigned>(KB));
      const uint32_t tS = tmem_base + TS_COL + (g & 1) * KB + lane_off;
      const uint32_t tO = tmem_base + TO_COL + (c.n & 1) * HD + lane_off;
      if (!warp_wait(&s_full[g & 1], (g >> 1) & 1, abort_flag, err, 16)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t pk[32];
      float lb = 0.f;
      if (any) {
        uint32_t sa[32], sb[32];  // scores of keys 0..31 and 32..63 of the block
        tmem_ld32(tS, sa);
        tmem_ld32(tS + 32, sb);
        tmem_ld_wait();
        if (!full) {  // masked scores become -inf before the maximum and the exponentials
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (static_cast<unsigned>(i - lo) >= span) sa[i] = __float_as_uint(-INFINITY);
            if (static_cast<unsigned>(i + 32 - lo) >= span) sb[i] = __float_as_uint(-INFINITY);
          }
        }
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          mx[(i >> 1) & 3] = max3(mx[(i >> 1) & 3], __uint_as_float(sa[i]), __uint_as_float(sa[i + 1]));
          mx[((i >> 1) + 2) & 3] = max3(mx[((i >> 1) + 2) & 3], __uint_as_float(sb[i]), __uint_as_float(sb[i + 1]));
        }
        const float bmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
        const bool moved = bmax > m_used + kRescaleLog2;  // also the row's first valid block
        const bool rescale = moved && m_used != -INFINITY;
        if (__any_sync(0xffffffffu, rescale)) {
          // O must be stable first: every P.V of this item issued so far has completed
          // (m_used is finite only after a block of this item, so g >= 1 here)
          if (!warp_wait(&pv_done[(g - 1) % NKV], ((g - 1) / NKV) & 1, abort_flag, err, 15)) ok = false;
          tc_fence_after();
          const float alpha = rescale ? ex2(m_used - bmax) : 1.f;
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
          l *= alpha;
        }
        if (moved) m_used = bmax;
        const float uu = (m_used == -INFINITY) ? 0.f : m_used;
        // pairs of keys: one packed FMA for both exponents, one packed add into the sums
        const uint64_t sc2 = f2pack(scale_log2, scale_log2), nu2 = f2pack(-uu, -uu);
        uint64_t lp2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t s0 = i < 16 ? sa[2 * i] : sb[2 * i - 32];
          const uint32_t s1 = i < 16 ? sa[2 * i + 1] : sb[2 * i - 31];
          float a0, a1;
          f2unpack(fma2(f2pack(__uint_as_float(s0), __uint_as_float(s1)), sc2, nu2), a0, a1);
          const float p0 = ex2(a0), p1 = ex2(a1);
          lp2[i & 3] = add2(lp2[i & 3], f2pack(p0, p1));
          pk[i] = pack_bf16x2(p0, p1);
        }
        float lq[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) f2unpack(lp2[k], lq[2 * k], lq[2 * k + 1]);
        lb = ((lq[0] + lq[1]) + (lq[2] + lq[3])) + ((lq[4] + lq[5]) + (lq[6] + lq[7]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) pk[i] = 0u;
      }
      release_q();  // the store issued during the previous block has had that block to read
      // P(g) overwrites S(g) in place: this thread's scores are in registers, and the MMA
      // issues nothing into these columns before P(g).V(g) has completed
      tmem_st32(tS, pk);
      tmem_st_wait();
      if (!ok) break;
      l += lb;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g & 1]);
      if (pend.on) {  // previous item's O: final once its o_full fires
        if (!warp_wait(&o_full[pend.n & 1], (pend.n >> 1) & 1, abort_flag, err, 18)) {
          ok = false;
          break;
        }
        tc_fence_after();
        epilogue();
      }
      if (c.j + 1 == it.nb) pend = {true, l, it.tl.q_row0, it.tl.nq, it.head, c.n};
      cursor_next(c, tiles, ntiles, items, window);
    }
    if (ok && pend.on) {
      if (warp_wait(&o_full[pend.n & 1], (pend.n >> 1) & 1, abort_flag, err, 18)) {
        tc_fence_after();
        epilogue();
      }
    }
    release_q();
    if (lane == 0) bulk_wait_all();  // no store of ours may still read smem at exit
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem_base, 256);
}

}  // namespace

int attention_pair_queries() { return QT; }
int attention_kv_box_rows() { return KB; }

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
  return static_cast<int>(launch_kernel(attn_tc_kernel, dim3(grid), dim3(192), ATT_SMEM, stream, tmQ, tmKV,
                                        tmO ? *tmO : tmQ, tmO ? 1 : 0, tiles, ntiles, heads, out, ldo, q_col0, k_col0,
                                        v_col0, window, scale_log2, err));
}

}  // namespace j1rt
