// Varlen FlashAttention-style kernel on tcgen05 / TMEM for head_dim 64.
//
// Replaces the reference's mma.sync kernel `attention_impl` (src/cuda/kernels.cu:272-391)
// with the same semantics: packed sequences without padding, per-(tile, head)
// online softmax in base 2 with scale 0.125*log2(e), an optional |i - j| <= window
// band (local layers, kernels.cu:304-308,332) and P rounded to BF16 before P.V.
// RoPE is not applied here: the Wqkv GEMM epilogue already rotated q and k.
//
// One CTA = one 128-query tile of one sequence x one head. 192 threads:
//   warps 0..3  softmax: thread r owns query row r (TMEM lane r); reads S from
//               TMEM, writes P (bf16, 128B-swizzled, K-major) to smem, keeps the
//               running O (64 fp32) in registers
//   warp 4      tcgen05.mma issuer: S = Q K^T (M=128, N=128, K=64) and
//               O_j = P_j V_j (M=128, N=64, K=128; V read MN-major)
//   warp 5      TMA producer: Q once, then K/V blocks of 128 keys
// TMEM: S in columns [0,128), O_j in [128,192).
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
constexpr uint32_t ATT_SMEM = 3 * TILE_BYTES + P_BYTES + 1024 + 256;

__global__ void __launch_bounds__(192, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                   const AttnTile* __restrict__ tiles, bf16* __restrict__ out, int ldo, int q_col0, int k_col0,
                   int v_col0, int window, float scale_log2, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + TILE_BYTES;
  uint8_t* sV = sK + TILE_BYTES;
  uint8_t* sP = sV + TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_free = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* p_full = bars + 4;
  uint64_t* o_full = bars + 5;
  uint64_t* drain = bars + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  const AttnTile tl = tiles[blockIdx.x];
  const int head = blockIdx.y;
  int kbeg = 0, kend = tl.kv_len;
  if (window >= 0) {
    kbeg = max(0, tl.q_pos0 - window);
    kend = min(tl.kv_len, tl.q_pos0 + tl.nq + window);
  }
  const int nblk = (kend - kbeg + KB - 1) / KB;
  {  // exit before allocating anything when an earlier CTA of this launch gave up
    __shared__ int s_abort;
    if (threadIdx.x == 0) s_abort = device_aborted(err) ? 1 : 0;
    __syncthreads();
    if (s_abort) return;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(kv_full, 1);
    mbar_init(kv_free, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 128);
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
  const uint32_t tS = tmem_base, tO = tmem_base + 128;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, TILE_BYTES);
      tma_load_2d(&tmQ, q_full, sQ, q_col0 + head * HD, tl.q_row0);
      uint32_t armed_kv = 0;  // parity+1 of the last armed kv phase (0 = none)
      for (int j = 0; j < nblk; ++j) {
        if (j > 0 && !mbar_wait(kv_free, (j - 1) & 1, abort_flag, err, 11)) break;
        mbar_arrive_expect_tx(kv_full, 2 * TILE_BYTES);
        const int krow = tl.kv_row0 + kbeg + j * KB;
        tma_load_2d(&tmKV, kv_full, sK, k_col0 + head * HD, krow);
        tma_load_2d(&tmKV, kv_full, sV, v_col0 + head * HD, krow);
        armed_kv = 1 + (j & 1);
      }
      if (*abort_flag) {
        volatile int no_abort = 0;
        mbar_wait(q_full, 0, &no_abort, nullptr, 0);
        if (armed_kv) mbar_wait(kv_full, armed_kv - 1, &no_abort, nullptr, 0);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t idO = idesc_bf16(128, 64, false, true);
      const uint32_t q0 = smem_u32(sQ), k0 = smem_u32(sK), v0 = smem_u32(sV), p0 = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, abort_flag, err, 12);
      for (int j = 0; j < nblk && ok; ++j) {
        if (!mbar_wait(kv_full, j & 1, abort_flag, err, 13)) break;
        // S_j overwrites TMEM S: P_{j-1} (written after S_{j-1} was read) must be complete.
        if (j > 0 && !mbar_wait(p_full, (j - 1) & 1, abort_flag, err, 14)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tS, sdesc_sw128(q0 + k * 32, 16, 1024), sdesc_sw128(k0 + k * 32, 16, 1024), idS, k > 0);
        umma_commit(s_full);
        // O_j = P_j V_j once P_j is in smem (and O_{j-1} has been read back).
        if (!mbar_wait(p_full, j & 1, abort_flag, err, 15)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < KB / 16; ++k) {
          const uint32_t pa = p0 + (k >> 2) * (QT * 128) + (k & 3) * 32;
          const uint32_t vb = v0 + k * 16 * 128;
          umma_bf16(tO, sdesc_sw128(pa, 16, 1024), sdesc_sw128(vb, 8192, 1024), idO, k > 0);
        }
        umma_commit(o_full);
        umma_commit(kv_free);
      }
      umma_commit(drain);
      volatile int no_abort = 0;
      mbar_wait(drain, 0, &no_abort, nullptr, 0);
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int r = threadIdx.x;  // query row == TMEM lane
    const int qpos = tl.q_pos0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    float m_run = -INFINITY;  // running max (scaled, base-2 domain)
    float l = 0.f;
    float u_prev = 0.f;       // max used for P_{j-1}
    float u_acc = -INFINITY;  // scale of o[]
    uint8_t* prow = sP + r * 128;
    const uint32_t sw = static_cast<uint32_t>(r & 7);
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      if (!mbar_wait(s_full, j & 1, abort_flag, err, 16)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int key0 = kbeg + j * KB;
      // pass 1: row max over the masked, scaled scores
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < KB / 32; ++c) {
        uint32_t sr[32];
        tmem_ld32(tS + lane_off + c * 32, sr);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = key0 + c * 32 + i;
          const bool valid = key < tl.kv_len && (window < 0 || abs(qpos - key) <= window);
          const float s = valid ? __uint_as_float(sr[i]) * scale_log2 : -INFINITY;
          mx = fmaxf(mx, s);
        }
      }
      const float m_new = fmaxf(m_run, mx);
      const float u = (m_new == -INFINITY) ? 0.f : m_new;
      l *= exp2f(m_run - u);
      m_run = m_new;
      // O_{j-1} must be read back before P_j overwrites the P buffer it was computed from.
      if (j > 0) {
        if (!mbar_wait(o_full, (j - 1) & 1, abort_flag, err, 17)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float a = exp2f(u_acc - u_prev);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t orr[32];
          tmem_ld32(tO + lane_off + h * 32, orr);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[h * 32 + i] = o[h * 32 + i] * a + __uint_as_float(orr[i]);
        }
        u_acc = u_prev;
      }
      // pass 2: P = exp2(s - u) as bf16 into the swizzled K-major P tile
#pragma unroll 1
      for (int c = 0; c < KB / 32; ++c) {
        uint32_t sr[32];
        tmem_ld32(tS + lane_off + c * 32, sr);
        tmem_ld_wait();
        float pv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = key0 + c * 32 + i;
          const bool valid = key < tl.kv_len && (window < 0 || abs(qpos - key) <= window);
          const float s = valid ? __uint_as_float(sr[i]) * scale_log2 : -INFINITY;
          pv[i] = exp2f(s - u);
          l += pv[i];
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
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
      u_prev = u;
    }
    if (ok && nblk > 0 && mbar_wait(o_full, (nblk - 1) & 1, abort_flag, err, 18)) {
      tc_fence_after();
      const float a = exp2f(u_acc - u_prev);
      const float inv = l > 0.f ? 1.f / l : 0.f;
      float res[HD];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t orr[32];
        tmem_ld32(tO + lane_off + h * 32, orr);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) res[h * 32 + i] = (o[h * 32 + i] * a + __uint_as_float(orr[i])) * inv;
      }
      if (r < tl.nq) {
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(tl.q_row0 + r) * ldo + head * HD);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          uint4 w;
          w.x = pack_bf16x2(res[8 * g + 0], res[8 * g + 1]);
          w.y = pack_bf16x2(res[8 * g + 2], res[8 * g + 3]);
          w.z = pack_bf16x2(res[8 * g + 4], res[8 * g + 5]);
          w.w = pack_bf16x2(res[8 * g + 6], res[8 * g + 7]);
          dst[g] = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem_base, 256);
}

}  // namespace

int launch_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, const AttnTile* tiles, int ntiles, int heads,
                     int q_col0, int k_col0, int v_col0, bf16* out, int ldo, int window, float scale_log2, int* err,
                     cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
  if (ntiles == 0 || heads == 0) return 0;
  dim3 grid(ntiles, heads);
  attn_tc_kernel<<<grid, 192, ATT_SMEM, stream>>>(tmQ, tmKV, tiles, out, ldo, q_col0, k_col0, v_col0, window,
                                                   scale_log2, err);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace j1rt
