// Host-side launch interface of the device kernels (internal to libj1).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <utility>

namespace j1rt {

using bf16 = __nv_bfloat16;

// Programmatic dependent launch for the forward's kernels: each is launched so that it may
// begin (launch its CTAs and run its local set-up: barriers, TMEM, descriptor prefetch) while
// the previous kernel of the stream drains, and waits (griddepcontrol.wait) before it reads or
// writes any global data. J1_PDL=0 in the environment launches them the ordinary way.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("J1_PDL");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// cudaFuncSetAttribute acts on the kernel as loaded in the current device's
// context, so a process that drives several GPUs (the engine pool) must raise the
// dynamic shared-memory limit once per device. `done` keeps one bit per device
// ordinal; ordinals of 64 and above set the attribute on every launch.
template <typename Kernel>
inline cudaError_t set_smem_once(Kernel kern, int bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev < 64 ? 1ull << dev : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// ------------------------------------------------------------------ GEMM
// out = A[M,K] . W[N,K]^T with a fused epilogue. A and W are bf16, row-major,
// read through 128B-swizzled TMA maps (box 64 x 128 for A, 64 x BN/2 for W: each CTA of a
// pair loads half of the tile's W rows; see gemm_w_box_rows).
enum GemmEpi : int {
  EPI_BF16 = 0,      // out = bf16(acc (+bias)) (relu when `relu`)
  EPI_QKV_ROPE = 1,  // out = bf16(rope(bf16(acc))) on columns < rope_cols, bf16(acc) elsewhere
  EPI_GEGLU = 2,     // W rows interleaved per 128: out[:, n/2 + j] = bf16(gelu(bf16(acc_a)) * bf16(acc_b))
  EPI_RESID_LN = 3,  // full row: x += bf16(acc) (+bias); xn = bf16(LN(x; ln_w, ln_b, eps))
  EPI_RESID = 4,     // full row: x += bf16(acc) (+bias)
  EPI_SCORER = 5,    // full row: scores[r] = sum_j gelu(acc + bias[j]) * w2[j] + b2
};

struct EpiParams {
  int M, N, K;
  bf16* out;
  int ldo;
  const float* bias;
  int relu;
  float* x;
  int ldx;
  const float* ln_w;
  const float* ln_b;
  float ln_eps;
  bf16* xn;
  int ldxn;
  const int* pos;
  const float* rope_cos;  // [max_pos, 32]
  const float* rope_sin;
  int rope_cols;
  const float* w2;
  float b2;
  float* scores;
  int* err;  // device error word
};

// Column width of one MMA tile for an N (or full-row width): 256 when N % 256 == 0, else 128.
int gemm_bn_for(int n);
// Rows of one W box for tile width bn (the two CTAs of a pair each load half of the tile).
inline uint32_t gemm_w_box_rows(int bn) { return static_cast<uint32_t>(bn / 2); }
// Returns 0 on success, or a cudaError_t value. tmX: the map of the epilogue's global tensor:
// the FP32 residual map (make_tmap_f32_resid, 32 x 128 boxes) over p.x for EPI_RESID_LN /
// EPI_RESID; the BF16 output map over p.out (make_tmap_bf16, box 64 x 128, N columns -- N/2
// for GEGLU -- and row stride p.ldo) for EPI_BF16 / EPI_QKV_ROPE / EPI_GEGLU; ignored by
// EPI_SCORER.
// For EPI_RESID_LN / EPI_RESID also: tmXs, the FP32 residual map over p.x with 32-row boxes
// (make_tmap_f32_resid(..., 32)) through which each epilogue warp stores its rows; and for
// EPI_RESID_LN tmXN, the BF16 map over p.xn with 64 x 32 boxes (make_tmap_bf16, N columns,
// row stride p.ldxn) through which the normalised rows leave.
int launch_gemm(GemmEpi epi, int bn, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap* tmX,
                const EpiParams& p, int grid_limit, cudaStream_t stream, const CUtensorMap* tmXs = nullptr,
                const CUtensorMap* tmXN = nullptr);
// EPI_RESID_LN (ln) / EPI_RESID on clusters of CTA pairs (gemm_resid.cu): x += bf16(A W^T)
// (+ bias); with ln, xn = bf16(LN(x)) through tmXN. N (= the hidden width) in {256, 384, 512,
// 768, 1024}; tmW boxes of gemm_w_box_rows(gemm_bn_for(N)) rows; tmX (loads) 32 x 128 boxes,
// tmXs (stores) 32 x 32 boxes, tmXN 64 x 32 boxes.
int launch_resid_gemm(bool ln, const CUtensorMap& tmA, const CUtensorMap& tmW, const CUtensorMap& tmX,
                      const CUtensorMap* tmXs, const CUtensorMap* tmXN, const EpiParams& p, int grid_limit,
                      cudaStream_t stream);
// Validates shapes for an epilogue; returns nullptr when fine, else a message.
const char* gemm_shape_error(GemmEpi epi, int bn, int M, int N, int K);

// ------------------------------------------------------------------ attention
// Queries covered by one attention work item (one 128-query tile).
int attention_pair_queries();
// Rows of one K/V box: the tmKV map given to launch_attention uses boxes of 64 x this.
int attention_kv_box_rows();
// One CTA's queries (up to attention_pair_queries()) of one sequence. Query row r of the tile is Q-buffer row
// q_row0 + r at sequence position q_pos0 + r; keys/values are rows
// kv_row0 .. kv_row0 + kv_len - 1 of the K/V buffer.
struct AttnTile {
  int q_row0, nq, kv_row0, kv_len, q_pos0, pad0, pad1, pad2;
};
// ctx[q_row0 + r, head*64 ..] = softmax(scale * q k^T [band]) v for every tile x head.
// tmQ: bf16 map with 64 x 128 boxes; tmKV: 64 x attention_kv_box_rows() boxes.
// window < 0: full attention; else |qpos - kpos| <= window.
// tmO (optional): bf16 map over out with 64 x 32 boxes (make_tmap_bf16(..., box_rows 32));
// full 32-row slices of O leave through it by TMA store, the rest by plain stores.
// Persistent: min(ntiles * heads, 2 * grid_limit) CTAs walk the (tile, head) items.
int launch_attention(const CUtensorMap& tmQ, const CUtensorMap& tmKV, const CUtensorMap* tmO, const AttnTile* tiles,
                     int ntiles, int heads, int q_col0, int k_col0, int v_col0, bf16* out, int ldo, int window,
                     float scale_log2, int* err, int grid_limit, cudaStream_t stream);

// ------------------------------------------------------------------ row kernels
int launch_embed_ln(int hidden, const int* ids, const float* table, const float* w, float* x, bf16* xn, int rows,
                    float eps, cudaStream_t stream);
int launch_final_norm(int hidden, float* x, const float* fw, const float* type_emb, const int* qtype_tok,
                      const float* hw, const float* hb, bf16* xn, int rows, float eps, cudaStream_t stream);
int launch_gather_rows(const void* src, const int* idx, void* dst, int rows, int row_bytes, cudaStream_t stream);
// dst = bf16(src) with an optional row permutation: dst row r <- src row perm(r) (GEGLU interleave).
int launch_f32_to_bf16(const float* src, bf16* dst, long long rows, int cols, int geglu_inter, cudaStream_t stream);
bool hidden_supported(int hidden);
// Self-test of the bounded device waits: one thread waits (with a limit of `limit` cycles) on an
// mbarrier nothing arrives at, records the timeout in *err and returns.
int launch_wait_timeout_selftest(int* err, long long limit, cudaStream_t stream);

// ------------------------------------------------------------------ TMA maps
// 2D bf16 row-major [rows, cols] with row stride `ld` elements; 128B swizzle box (64 x box_rows).
bool make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                    uint32_t box_rows, const char** why);
// 2D fp32 row-major residual [rows, cols] (row stride `ld` elements); 128B-swizzled 32 x 128 box.
bool make_tmap_f32_resid(CUtensorMap* map, const float* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         const char** why, uint32_t box_rows = 128);

}  // namespace j1rt
