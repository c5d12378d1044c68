// CudaModel equivalent: weight upload, workspace, batch staging and the forward
// launch sequence (src/cuda/mod.rs:174-521), plus the kernel-level op entry points.
#include "model.h"

#include <sys/stat.h>

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <system_error>
#include <thread>
#include <unordered_map>

namespace j1rt {

namespace {
thread_local std::string t_last_error;

constexpr float kScaleLog2 = 0.125f * 1.44269504088896340736f;  // 1/sqrt(64) * log2(e), src/cuda/mod.rs:391

size_t copy_out(const std::string& s, char* buf, size_t cap) {
  if (buf && cap) {
    const size_t n = s.size() < cap - 1 ? s.size() : cap - 1;
    std::memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return s.size();
}

bool file_exists(const std::string& p) {
  struct stat st;
  return ::stat(p.c_str(), &st) == 0;
}

size_t next_pow2(size_t v) {
  size_t p = 1;
  while (p < v) p <<= 1;
  return p;
}
}  // namespace

j1_status set_error(j1_status s, const std::string& msg) {
  t_last_error = msg;
  return s;
}

j1_status set_error_noexcept(j1_status s, const char* fn, const char* what) noexcept {
  try {
    t_last_error = std::string(fn) + ": " + what;
  } catch (...) {
    t_last_error.clear();
  }
  return s;
}

void run_pool(int n, const std::function<void()>& work) {
  std::exception_ptr first;
  std::mutex mu;
  auto safe = [&]() noexcept {
    try {
      if (take_fault(J1_FAULT_WORKER)) throw std::runtime_error("injected worker failure");
      work();
    } catch (...) {
      std::lock_guard<std::mutex> lock(mu);
      if (!first) first = std::current_exception();
    }
  };
  std::vector<std::thread> pool;
  for (int k = 1; k < n; ++k) {
    try {
      if (take_fault(J1_FAULT_THREAD)) throw std::system_error(std::make_error_code(std::errc::resource_unavailable_try_again));
      pool.emplace_back(safe);
    } catch (...) {  // no thread (or no room to hold one): the started ones and this thread do the rest
      break;
    }
  }
  safe();
  for (auto& th : pool) th.join();
  if (first) std::rethrow_exception(first);
}

j1_status cuda_error(cudaError_t e, const char* what) {
  if (e == cudaErrorMemoryAllocation) return set_error(J1_ERR_OOM, std::string(what) + ": out of device memory");
  return set_error(J1_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

size_t last_error_copy(char* buf, size_t cap) { return copy_out(t_last_error, buf, cap); }

// Host-side fault injection (j1_inject_fault, or J1_FAULT=alloc|launch|nan at model
// creation): the next `count` device allocations / kernel launches / score readbacks of
// the process report a failure, so callers can test their error handling. Nothing is done
// to the GPU: an injected allocation or launch simply does not happen, and injected
// nonfinite scores are written into the host copy.
std::atomic<int> g_fault[8];

bool take_fault(int kind) {
  int n = g_fault[kind].load();
  while (n > 0)
    if (g_fault[kind].compare_exchange_weak(n, n - 1)) return true;
  return false;
}

bool fault_pending(int kind) { return g_fault[kind].load() > 0; }

}  // namespace j1rt

using namespace j1rt;

namespace {

#define J1_TRY_CUDA(expr, what)                          \
  do {                                                   \
    cudaError_t e_ = (expr);                             \
    if (e_ != cudaSuccess) return cuda_error(e_, what);  \
  } while (0)

// Kernel families for j1_model_profile (order of j1_profile_family_name).
enum Family {
  F_EMBED = 0, F_QKV, F_ATTN_LOCAL, F_ATTN_GLOBAL, F_WO, F_WI, F_WO2, F_FINAL, F_HEAD_GEMM, F_HEAD_ATTN,
  F_HEAD_ROWS, F_SCORER
};
const char* const kFamilyNames[J1_PROF_FAMILIES] = {
    "embed_ln", "gemm_qkv_rope", "attn_local", "attn_global", "gemm_wo_resid_ln", "gemm_wi_geglu",
    "gemm_wo2_resid_ln", "final_norm", "head_gemm", "head_attn", "head_gather", "scorer_gemm"};

cudaEvent_t* prof_slot(j1_model* model, int fam) {
  const size_t need = 2 * (model->prof_used + 1);
  while (model->prof_ev.size() < need) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    model->prof_ev.push_back(e);
  }
  if (model->prof_fam.size() < model->prof_used + 1) model->prof_fam.resize(model->prof_used + 1);
  model->prof_fam[model->prof_used] = fam;
  return &model->prof_ev[2 * model->prof_used++];
}

void prof_fold(j1_model* model) {
  for (size_t i = 0; i < model->prof_used; ++i) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, model->prof_ev[2 * i], model->prof_ev[2 * i + 1]) == cudaSuccess) {
      model->prof_ms[model->prof_fam[i]] += ms;
      model->prof_cnt[model->prof_fam[i]] += 1;
    }
  }
  model->prof_used = 0;
}

// One launch: an NVTX range named by its kernel family (profilers), optional per-family
// CUDA-event timing (j1_model_profile), injected launch faults.
#define J1_TRY_LAUNCH(fam, expr, what)                                                       \
  do {                                                                                       \
    if (take_fault(J1_FAULT_LAUNCH)) return set_error(J1_ERR_CUDA, std::string(what) + ": injected launch failure"); \
    cudaEvent_t* ev_ = model->prof_on ? prof_slot(model, (fam)) : nullptr;                   \
    nvtxRangePushA(j1_profile_family_name(fam));                                             \
    if (ev_) cudaEventRecord(ev_[0], model->stream);                                         \
    int rc_ = (expr);                                                                        \
    if (ev_) cudaEventRecord(ev_[1], model->stream);                                         \
    nvtxRangePop();                                                                          \
    if (rc_ != 0) return cuda_error(static_cast<cudaError_t>(rc_), what);                    \
    ++model->launches;                                                                       \
  } while (0)

j1_status dalloc(j1_model* model, void** p, size_t bytes, std::vector<void*>& list) {
  *p = nullptr;
  if (take_fault(J1_FAULT_ALLOC)) return set_error(J1_ERR_OOM, "cudaMalloc: out of device memory (injected)");
  cudaError_t e = cudaMalloc(p, bytes < 256 ? 256 : bytes);
  if (e != cudaSuccess) return cuda_error(e, "cudaMalloc");
  list.push_back(*p);
  (void)model;
  return J1_OK;
}

template <class T>
j1_status upload_f32(j1_model* model, SafeTensors& st, const std::string& name, const std::vector<size_t>& shape,
                     T** out) {
  std::string err;
  const float* h = st.f32(name, shape, err);
  if (!h) return set_error(J1_ERR_IO, err);
  size_t n = 1;
  for (size_t d : shape) n *= d;
  void* p;
  j1_status s = dalloc(model, &p, n * 4, model->allocations);
  if (s) return s;
  // Ordered on the model's stream: a pageable cudaMemcpy may return before its DMA lands,
  // and the model's non-blocking stream would not wait for it.
  J1_TRY_CUDA(cudaMemcpyAsync(p, h, n * 4, cudaMemcpyHostToDevice, model->stream), "weight upload");
  J1_TRY_CUDA(cudaStreamSynchronize(model->stream), "weight upload");
  *out = static_cast<T*>(p);
  return J1_OK;
}

// GEMM weight: F32 on disk -> BF16 on device (round-to-nearest-even, as half::bf16::from_f32
// in src/cuda/mod.rs:36-39), optionally with the GEGLU row interleave; plus its TMA map.
j1_status upload_bf16(j1_model* model, SafeTensors& st, const std::string& name, size_t rows, size_t cols,
                      int geglu_inter, float* staging, bf16** out, CUtensorMap* tm, uint32_t tile_n) {
  std::string err;
  const float* h = st.f32(name, {rows, cols}, err);
  if (!h) return set_error(J1_ERR_IO, err);
  void* p;
  j1_status s = dalloc(model, &p, rows * cols * 2, model->allocations);
  if (s) return s;
  J1_TRY_CUDA(cudaMemcpyAsync(staging, h, rows * cols * 4, cudaMemcpyHostToDevice, model->stream), "weight upload");
  int rc = launch_f32_to_bf16(staging, static_cast<bf16*>(p), static_cast<long long>(rows), static_cast<int>(cols),
                              geglu_inter, model->stream);
  if (rc) return cuda_error(static_cast<cudaError_t>(rc), "weight conversion");
  J1_TRY_CUDA(cudaStreamSynchronize(model->stream), "weight conversion");
  *out = static_cast<bf16*>(p);
  const char* why = nullptr;
  if (!make_tmap_bf16(tm, p, rows, cols, cols, gemm_w_box_rows(static_cast<int>(tile_n)), &why))
    return set_error(J1_ERR_CUDA, std::string(name) + ": " + (why ? why : "tensor map"));
  return J1_OK;
}

void drop_forward_graphs(j1_model* model) {
  for (auto& g : model->graphs) cudaGraphExecDestroy(g.exec);
  model->graphs.clear();
  model->shapes_seen.clear();
}

void free_workspace(j1_model* model) {
  drop_forward_graphs(model);  // their kernels hold pointers into the workspace
  ++model->ws_gen;
  for (void* p : model->ws_allocations) cudaFree(p);
  model->ws_allocations.clear();
  for (int k = 0; k < 2; ++k) {
    if (model->meta_host[k]) cudaFreeHost(model->meta_host[k]);
    if (model->scores_host[k]) cudaFreeHost(model->scores_host[k]);
    model->meta_host[k] = nullptr;
    model->scores_host[k] = nullptr;
    model->meta_dev[k] = nullptr;
    model->slot_busy[k] = false;
  }
  model->cap_tokens = model->cap_markers = model->cap_meta = 0;
}

j1_status ensure_workspace(j1_model* model, size_t tokens, size_t markers, size_t meta_ints) {
  const ModelConfig& c = model->cfg;
  const size_t H = c.hidden, I = c.intermediate, FF = c.head_ff;
  if (tokens > model->cap_tokens || markers > model->cap_markers || meta_ints > model->cap_meta) {
    J1_TRY_CUDA(cudaStreamSynchronize(model->stream), "workspace");
    size_t T = next_pow2(std::max(tokens, model->cap_tokens));
    if (T < 1024) T = 1024;
    size_t M = next_pow2(std::max(markers, model->cap_markers));
    if (M < 256) M = 256;
    size_t E = next_pow2(std::max(meta_ints, model->cap_meta));
    if (E < 16384) E = 16384;
    free_workspace(model);
    void* p;
    auto& L = model->ws_allocations;
    j1_status s;
#define J1_WS(field, type, bytes)                     \
  if ((s = dalloc(model, &p, (bytes), L))) return s;  \
  model->field = static_cast<type>(p);
    J1_WS(x, float*, T * H * 4)
    J1_WS(xn, bf16*, T * H * 2)
    J1_WS(qkv, bf16*, T * 3 * H * 2)
    J1_WS(ctx, bf16*, T * H * 2)
    J1_WS(g, bf16*, T * std::max(I, FF) * 2)
    J1_WS(ym, float*, M * H * 4)
    J1_WS(ymb, bf16*, M * H * 2)
    J1_WS(cm, bf16*, M * H * 2)
    J1_WS(hm, bf16*, M * FF * 2)
    J1_WS(qm, bf16*, M * H * 2)
    J1_WS(scores, float*, M * 4)
    J1_WS(meta_dev[0], int*, E * 4)
    J1_WS(meta_dev[1], int*, E * 4)
#undef J1_WS
    for (int k = 0; k < 2; ++k) {
      J1_TRY_CUDA(cudaMallocHost(&p, E * 4), "cudaMallocHost");
      model->meta_host[k] = static_cast<int*>(p);
      J1_TRY_CUDA(cudaMallocHost(&p, M * 4), "cudaMallocHost");
      model->scores_host[k] = static_cast<float*>(p);
    }
    model->cap_tokens = T;
    model->cap_markers = M;
    model->cap_meta = E;
  }
  return J1_OK;
}

j1_status validate_batch(const j1_model* model, const BatchView& b) {
  const ModelConfig& c = model->cfg;
  if (b.t && !b.ids) return set_error(J1_ERR_INVALID_ARG, "ids is NULL");
  if (b.nseq && (!b.starts || !b.lens || !b.qtypes || !b.marker_starts))
    return set_error(J1_ERR_INVALID_ARG, "batch arrays are NULL");
  if (b.m && !b.marker_rows) return set_error(J1_ERR_INVALID_ARG, "marker_rows is NULL");
  if (b.t > (size_t(1) << 26)) return set_error(J1_ERR_INVALID_ARG, "batch too large (> 2^26 tokens)");
  size_t row = 0;
  for (size_t s = 0; s < b.nseq; ++s) {
    if (b.starts[s] != row) return set_error(J1_ERR_INVALID_ARG, "sequences must be packed back to back");
    if (b.lens[s] == 0) return set_error(J1_ERR_INVALID_ARG, "empty sequence in batch");
    if (b.lens[s] > static_cast<uint32_t>(c.max_positions))
      return set_error(J1_ERR_INVALID_ARG, "sequence longer than max_position_embeddings");
    if (b.qtypes[s] > 2) return set_error(J1_ERR_INVALID_ARG, "qtype must be 0, 1 or 2");
    row += b.lens[s];
  }
  if (row != b.t) return set_error(J1_ERR_INVALID_ARG, "sum of lens does not match t");
  if (b.nseq && b.marker_starts[0] != 0) return set_error(J1_ERR_INVALID_ARG, "marker_starts[0] must be 0");
  for (size_t s = 0; s < b.nseq; ++s) {
    const uint32_t a = b.marker_starts[s], e = b.marker_starts[s + 1];
    if (e < a || e > b.m) return set_error(J1_ERR_INVALID_ARG, "marker_starts must be non-decreasing and <= m");
    for (uint32_t k = a; k < e; ++k)
      if (b.marker_rows[k] < b.starts[s] || b.marker_rows[k] >= b.starts[s] + b.lens[s])
        return set_error(J1_ERR_INVALID_ARG, "marker row outside its sequence");
  }
  if (b.nseq && b.marker_starts[b.nseq] != b.m) return set_error(J1_ERR_INVALID_ARG, "marker_starts[nseq] != m");
  if (!b.nseq && (b.t || b.m)) return set_error(J1_ERR_INVALID_ARG, "tokens without sequences");
  for (size_t i = 0; i < b.t; ++i)
    if (b.ids[i] >= static_cast<uint32_t>(c.vocab)) return set_error(J1_ERR_INVALID_ARG, "token id out of vocabulary");
  return J1_OK;
}

// Layout of a batch's metadata (ints): ids[t] | pos[t] | qtype per token[t] | markers[m]
// | pad to 8 | attention tiles | marker-query tiles (8 ints per tile).
struct MetaLayout {
  size_t ntiles = 0, nmtiles = 0, tiles_off = 0, ints = 0;
};
MetaLayout meta_layout(const BatchView& b) {
  MetaLayout L;
  const int PQ = attention_pair_queries();  // queries per attention work item
  for (size_t q = 0; q < b.nseq; ++q) {
    L.ntiles += (b.lens[q] + PQ - 1) / PQ;
    L.nmtiles += (b.marker_starts[q + 1] - b.marker_starts[q] + PQ - 1) / PQ;
  }
  L.tiles_off = (3 * b.t + b.m + 7) / 8 * 8;
  L.ints = L.tiles_off + (L.ntiles + L.nmtiles) * 8;
  return L;
}

// Packs a validated batch into staging slot `slot` and uploads it (async, model stream).
// The slot's pinned buffer may only be rewritten once its previous use has completed:
// with `sync` the whole stream is drained first (single-batch calls), otherwise the
// slot's completion event is awaited (pipelined calls).
j1_status stage_batch(j1_model* model, const BatchView& b, int slot = 0, bool sync = true) {
  j1_status s = validate_batch(model, b);
  if (s) return s;
  if (sync) J1_TRY_CUDA(cudaStreamSynchronize(model->stream), "stage");
  else if (model->slot_busy[slot]) J1_TRY_CUDA(cudaEventSynchronize(model->slot_done[slot]), "stage");
  const MetaLayout L = meta_layout(b);
  const size_t ntiles = L.ntiles, nmtiles = L.nmtiles, tiles_off = L.tiles_off, meta_ints = L.ints;
  const int PQ = attention_pair_queries();
  const size_t t = b.t, m = b.m;
  if ((s = ensure_workspace(model, t, m, meta_ints))) return s;
  int* h = model->meta_host[slot];
  for (size_t i = 0; i < t; ++i) h[i] = static_cast<int>(b.ids[i]);
  size_t o = 0;
  AttnTile* tiles = reinterpret_cast<AttnTile*>(h + tiles_off);
  size_t ti = 0;
  for (size_t q = 0; q < b.nseq; ++q) {
    const int start = static_cast<int>(b.starts[q]), len = static_cast<int>(b.lens[q]);
    for (int p = 0; p < len; ++p) {
      h[t + o] = p;                           // position within the sequence
      h[2 * t + o] = static_cast<int>(b.qtypes[q]);  // per-token qtype (src/cuda/mod.rs:428-432)
      ++o;
    }
    for (int q0 = 0; q0 < len; q0 += PQ) {
      AttnTile& tl = tiles[ti++];
      tl.q_row0 = start + q0;
      tl.nq = len - q0 < PQ ? len - q0 : PQ;
      tl.kv_row0 = start;
      tl.kv_len = len;
      tl.q_pos0 = q0;
      tl.pad0 = tl.pad1 = tl.pad2 = 0;
    }
  }
  // last head layer: the marker rows of each sequence as query tiles (rows of qm) over
  // all of that sequence's keys
  for (size_t q = 0; q < b.nseq; ++q) {
    const int k0 = static_cast<int>(b.marker_starts[q]), k1 = static_cast<int>(b.marker_starts[q + 1]);
    for (int r0 = k0; r0 < k1; r0 += PQ) {
      AttnTile& tl = tiles[ti++];
      tl.q_row0 = r0;
      tl.nq = k1 - r0 < PQ ? k1 - r0 : PQ;
      tl.kv_row0 = static_cast<int>(b.starts[q]);
      tl.kv_len = static_cast<int>(b.lens[q]);
      tl.q_pos0 = 0;
      tl.pad0 = tl.pad1 = tl.pad2 = 0;
    }
  }
  for (size_t k = 0; k < m; ++k) h[3 * t + k] = static_cast<int>(b.marker_rows[k]);
  if (meta_ints)
    J1_TRY_CUDA(cudaMemcpyAsync(model->meta_dev[slot], h, meta_ints * 4, cudaMemcpyHostToDevice, model->stream),
                "meta upload");
  model->slot = slot;
  model->t = t;
  model->m = m;
  model->nseq = b.nseq;
  model->ntiles = ntiles;
  model->nmtiles = nmtiles;
  int* md = model->meta_dev[slot];
  model->d_ids = md;
  model->d_pos = md + t;
  model->d_qtype = md + 2 * t;
  model->d_markers = md + 3 * t;
  model->d_tiles = reinterpret_cast<AttnTile*>(md + tiles_off);
  model->d_mtiles = model->d_tiles + ntiles;
  const ModelConfig& c = model->cfg;
  const size_t H = c.hidden, I = c.intermediate, FF = c.head_ff;
  const char* why = nullptr;
  bool ok = make_tmap_bf16(&model->tm_xn, model->xn, t, H, H, 128, &why) &&
            make_tmap_bf16(&model->tm_ctx, model->ctx, t, H, H, 128, &why) &&
            make_tmap_bf16(&model->tm_g, model->g, t, I, I, 128, &why) &&
            make_tmap_bf16(&model->tm_h, model->g, t, FF, FF, 128, &why) &&
            make_tmap_bf16(&model->tm_qkv, model->qkv, t, 3 * H, 3 * H, 128, &why) &&
            make_tmap_bf16(&model->tm_cm, model->cm, m, H, H, 128, &why) &&
            make_tmap_bf16(&model->tm_ymb, model->ymb, m, H, H, 128, &why) &&
            make_tmap_bf16(&model->tm_hm, model->hm, m, FF, FF, 128, &why) &&
            make_tmap_bf16(&model->tm_qm, model->qm, m, H, H, 128, &why) &&
            make_tmap_bf16(&model->tm_ctx_o, model->ctx, t, H, H, 32, &why) &&
            make_tmap_bf16(&model->tm_kv, model->qkv, t, 3 * H, 3 * H, attention_kv_box_rows(), &why) &&
            make_tmap_bf16(&model->tm_cm_o, model->cm, m, H, H, 32, &why) &&
            make_tmap_f32_resid(&model->tm_x, model->x, t, H, H, &why) &&
            make_tmap_f32_resid(&model->tm_ym, model->ym, m, H, H, &why) &&
            make_tmap_f32_resid(&model->tm_x_st, model->x, t, H, H, &why, 32) &&
            make_tmap_f32_resid(&model->tm_ym_st, model->ym, m, H, H, &why, 32) &&
            make_tmap_bf16(&model->tm_xn_st, model->xn, t, H, H, 32, &why) &&
            make_tmap_bf16(&model->tm_ymb_st, model->ymb, m, H, H, 32, &why) &&
            make_tmap_bf16(&model->tm_qkv_kv, model->qkv + H, t, 2 * H, 3 * H, 128, &why);
  if (!ok) return set_error(J1_ERR_CUDA, std::string("activation tensor map: ") + (why ? why : ""));
  model->staged = true;
  return J1_OK;
}

j1_status launch_forward_direct(j1_model* model) {
  if (!model->staged) return set_error(J1_ERR_INVALID_ARG, "no staged batch");
  const ModelConfig& c = model->cfg;
  const int H = c.hidden, I = c.intermediate, FF = c.head_ff, L = c.layers;
  const int t = static_cast<int>(model->t), m = static_cast<int>(model->m);
  const int nsm = model->num_sms;
  cudaStream_t st = model->stream;
  model->launches = 0;
  if (t == 0) return J1_OK;
  const int bn_full = gemm_bn_for(H), bn_qkv = gemm_bn_for(3 * H), bn_ff = gemm_bn_for(FF);
  EpiParams base;
  std::memset(&base, 0, sizeof(base));
  base.err = model->err_dev;

  J1_TRY_LAUNCH(F_EMBED, launch_embed_ln(H, model->d_ids, model->emb, model->emb_norm, model->x, model->xn, t, c.norm_eps, st),
                "embed_ln");
  for (int l = 0; l < L; ++l) {
    const auto& ly = model->layers[l];
    EpiParams p = base;
    p.M = t, p.N = 3 * H, p.K = H;
    p.out = model->qkv, p.ldo = 3 * H;
    p.pos = model->d_pos, p.rope_cos = model->rope_cos[ly.rope], p.rope_sin = model->rope_sin[ly.rope];
    p.rope_cols = 2 * H;
    J1_TRY_LAUNCH(F_QKV, launch_gemm(EPI_QKV_ROPE, bn_qkv, model->tm_xn, ly.tm_wqkv, &model->tm_qkv, p, nsm, st), "gemm qkv");
    J1_TRY_LAUNCH(ly.global ? F_ATTN_GLOBAL : F_ATTN_LOCAL,
                  launch_attention(model->tm_qkv, model->tm_kv, &model->tm_ctx_o, model->d_tiles, static_cast<int>(model->ntiles),
                                   c.heads, 0, H, 2 * H, model->ctx, H, ly.global ? -1 : c.half_window, kScaleLog2,
                                   model->err_dev, nsm, st),
                  "attention");
    p = base;
    p.M = t, p.N = H, p.K = H;
    p.x = model->x, p.ldx = H;
    p.ln_w = ly.mlp_norm, p.ln_eps = c.norm_eps, p.xn = model->xn, p.ldxn = H;
    J1_TRY_LAUNCH(F_WO, launch_gemm(EPI_RESID_LN, bn_full, model->tm_ctx, ly.tm_wo, &model->tm_x, p, nsm, st, &model->tm_x_st, &model->tm_xn_st), "gemm wo");
    p = base;
    p.M = t, p.N = 2 * I, p.K = H;
    p.out = model->g, p.ldo = I;
    J1_TRY_LAUNCH(F_WI, launch_gemm(EPI_GEGLU, 256, model->tm_xn, ly.tm_wi, &model->tm_g, p, nsm, st), "gemm wi");
    p = base;
    p.M = t, p.N = H, p.K = I;
    p.x = model->x, p.ldx = H;
    if (l + 1 < L) {
      p.ln_w = model->layers[l + 1].attn_norm, p.ln_eps = c.norm_eps, p.xn = model->xn, p.ldxn = H;
      J1_TRY_LAUNCH(F_WO2, launch_gemm(EPI_RESID_LN, bn_full, model->tm_g, ly.tm_wo2, &model->tm_x, p, nsm, st, &model->tm_x_st, &model->tm_xn_st), "gemm wo2");
    } else {
      J1_TRY_LAUNCH(F_WO2, launch_gemm(EPI_RESID, bn_full, model->tm_g, ly.tm_wo2, &model->tm_x, p, nsm, st, &model->tm_x_st), "gemm wo2");
    }
  }
  const auto& h0 = model->head[0];
  J1_TRY_LAUNCH(F_FINAL, launch_final_norm(H, model->x, model->final_norm, model->type_emb, model->d_qtype, h0.norm1_w,
                                  h0.norm1_b, model->xn, t, c.norm_eps, st),
                "final_norm");
  const int nh = static_cast<int>(model->head.size());
  for (int j = 0; j < nh; ++j) {
    const auto& hl = model->head[j];
    EpiParams p = base;
    if (j + 1 < nh) {
      p.M = t, p.N = 3 * H, p.K = H;
      p.bias = hl.in_b;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_BF16, bn_qkv, model->tm_xn, hl.tm_in, &model->tm_qkv, p, nsm, st), "gemm in_proj");
      J1_TRY_LAUNCH(F_HEAD_ATTN,
                    launch_attention(model->tm_qkv, model->tm_kv, &model->tm_ctx_o, model->d_tiles, static_cast<int>(model->ntiles),
                                     c.head_heads, 0, H, 2 * H, model->ctx, H, -1, kScaleLog2, model->err_dev, nsm, st),
                    "head attention");
      p = base;
      p.M = t, p.N = H, p.K = H, p.bias = hl.out_b;
      p.x = model->x, p.ldx = H, p.ln_w = hl.norm2_w, p.ln_b = hl.norm2_b, p.ln_eps = 1e-5f;
      p.xn = model->xn, p.ldxn = H;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_RESID_LN, bn_full, model->tm_ctx, hl.tm_out, &model->tm_x, p, nsm, st, &model->tm_x_st, &model->tm_xn_st), "gemm out_proj");
      p = base;
      p.M = t, p.N = FF, p.K = H, p.bias = hl.lin1_b, p.relu = 1;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_BF16, bn_ff, model->tm_xn, hl.tm_lin1, &model->tm_h, p, nsm, st), "gemm linear1");
      const auto& nx = model->head[j + 1];
      p = base;
      p.M = t, p.N = H, p.K = FF, p.bias = hl.lin2_b;
      p.x = model->x, p.ldx = H, p.ln_w = nx.norm1_w, p.ln_b = nx.norm1_b, p.ln_eps = 1e-5f;
      p.xn = model->xn, p.ldxn = H;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_RESID_LN, bn_full, model->tm_h, hl.tm_lin2, &model->tm_x, p, nsm, st, &model->tm_x_st, &model->tm_xn_st), "gemm linear2");
    } else if (m > 0) {
      // Last head layer: only the option markers feed the scorer, so the queries, the
      // attention rows and everything after them are computed for the m marker rows
      // alone (the reference's CPU path does the same, src/cpu/mod.rs:293-321; its CUDA
      // path computes all t rows and gathers, src/cuda/mod.rs:480-507 -- rows are
      // independent, so the marker rows agree). Keys and values still cover every token.
      J1_TRY_LAUNCH(F_HEAD_ROWS, launch_gather_rows(model->xn, model->d_markers, model->ymb, m, H * 2, st), "gather xn");
      p.M = m, p.N = H, p.K = H, p.bias = hl.in_b;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_BF16, bn_full, model->tm_ymb, hl.tm_in_q, &model->tm_qm, p, nsm, st), "gemm in_proj q");
      p = base;
      p.M = t, p.N = 2 * H, p.K = H, p.bias = hl.in_b + H;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_BF16, gemm_bn_for(2 * H), model->tm_xn, hl.tm_in_kv, &model->tm_qkv_kv, p, nsm, st), "gemm in_proj kv");
      J1_TRY_LAUNCH(F_HEAD_ATTN,
                    launch_attention(model->tm_qm, model->tm_kv, &model->tm_cm_o, model->d_mtiles, static_cast<int>(model->nmtiles),
                                     c.head_heads, 0, H, 2 * H, model->cm, H, -1, kScaleLog2, model->err_dev, nsm, st),
                    "head attention (markers)");
      J1_TRY_LAUNCH(F_HEAD_ROWS, launch_gather_rows(model->x, model->d_markers, model->ym, m, H * 4, st), "gather x");
      p = base;
      p.M = m, p.N = H, p.K = H, p.bias = hl.out_b;
      p.x = model->ym, p.ldx = H, p.ln_w = hl.norm2_w, p.ln_b = hl.norm2_b, p.ln_eps = 1e-5f;
      p.xn = model->ymb, p.ldxn = H;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_RESID_LN, bn_full, model->tm_cm, hl.tm_out, &model->tm_ym, p, nsm, st, &model->tm_ym_st, &model->tm_ymb_st), "gemm out_proj");
      p = base;
      p.M = m, p.N = FF, p.K = H, p.bias = hl.lin1_b, p.relu = 1;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_BF16, bn_ff, model->tm_ymb, hl.tm_lin1, &model->tm_hm, p, nsm, st), "gemm linear1");
      p = base;
      p.M = m, p.N = H, p.K = FF, p.bias = hl.lin2_b;
      p.x = model->ym, p.ldx = H, p.ln_w = model->s_norm_w, p.ln_b = model->s_norm_b, p.ln_eps = 1e-5f;
      p.xn = model->ymb, p.ldxn = H;
      J1_TRY_LAUNCH(F_HEAD_GEMM, launch_gemm(EPI_RESID_LN, bn_full, model->tm_hm, hl.tm_lin2, &model->tm_ym, p, nsm, st, &model->tm_ym_st, &model->tm_ymb_st), "gemm linear2");
    }
  }
  EpiParams p = base;
  p.M = m, p.N = H, p.K = H, p.bias = model->s_b1, p.w2 = model->s_w2, p.b2 = model->s_b2, p.scores = model->scores;
  J1_TRY_LAUNCH(F_SCORER, launch_gemm(EPI_SCORER, bn_full, model->tm_ymb, model->tm_s_w1, nullptr, p, nsm, st), "gemm scorer");
  return J1_OK;
}

// Queues the readback of the launched forward's scores and error word into the staged
// slot's pinned buffers and marks the slot's completion.
j1_status enqueue_readback(j1_model* model) {
  const int slot = model->slot;
  if (model->m)
    J1_TRY_CUDA(cudaMemcpyAsync(model->scores_host[slot], model->scores, model->m * 4, cudaMemcpyDeviceToHost,
                                model->stream),
                "scores readback");
  J1_TRY_CUDA(cudaMemcpyAsync(model->err_host + slot, model->err_dev, 4, cudaMemcpyDeviceToHost, model->stream),
              "error word readback");
  J1_TRY_CUDA(cudaEventRecord(model->slot_done[slot], model->stream), "event");
  model->slot_busy[slot] = true;
  return J1_OK;
}

bool graphs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("J1_GRAPH");
    return !(v && std::strcmp(v, "0") == 0);
  }();
  return on;
}

// The staged batch's forward: replayed from a CUDA graph when its shape has been captured,
// captured when the shape is launched for the second time, launched kernel by kernel
// otherwise (and while per-launch profiling or an injected launch failure is pending). A
// graph holds the same kernels with the same arguments as the direct launches (programmatic
// dependent launch edges included); it saves the host's per-kernel launch work and part of
// the gaps between kernels, which matters for small micro-batches.
j1_status launch_forward(j1_model* model) {
  if (!graphs_enabled() || !model->staged || model->prof_on || model->t == 0 || fault_pending(J1_FAULT_LAUNCH))
    return launch_forward_direct(model);
  const std::array<uint64_t, 7> key = {model->t, model->m, model->nseq, model->ntiles, model->nmtiles,
                                       static_cast<uint64_t>(model->slot), model->ws_gen};
  for (auto& g : model->graphs)
    if (std::equal(key.begin(), key.end(), g.key)) {
      J1_TRY_CUDA(cudaGraphLaunch(g.exec, model->stream), "forward graph launch");
      g.last_use = ++model->graph_tick;
      model->launches = g.launches;
      return J1_OK;
    }
  auto seen = std::find(model->shapes_seen.begin(), model->shapes_seen.end(), key);
  if (seen == model->shapes_seen.end()) {  // first time: launch directly, remember the shape
    if (model->shapes_seen.size() >= 16) model->shapes_seen.erase(model->shapes_seen.begin());
    model->shapes_seen.push_back(key);
    return launch_forward_direct(model);
  }
  model->shapes_seen.erase(seen);
  // Second time: capture the launch sequence (nothing runs while capturing), then replay it.
  J1_TRY_CUDA(cudaStreamBeginCapture(model->stream, cudaStreamCaptureModeThreadLocal), "forward graph capture");
  const j1_status s = launch_forward_direct(model);
  cudaGraph_t graph = nullptr;
  const cudaError_t ec = cudaStreamEndCapture(model->stream, &graph);
  if (s) {  // a launch failed while capturing: nothing was queued, report that launch's error
    if (graph) cudaGraphDestroy(graph);
    return s;
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t ei = ec;
  if (ec == cudaSuccess) ei = cudaGraphInstantiate(&exec, graph, 0);
  if (graph) cudaGraphDestroy(graph);
  if (ei != cudaSuccess) {  // no graph for this shape: run the forward directly
    (void)cudaGetLastError();
    return launch_forward_direct(model);
  }
  if (model->graphs.size() >= 8) {
    auto lru = std::min_element(model->graphs.begin(), model->graphs.end(),
                                [](const j1_model::ForwardGraph& a, const j1_model::ForwardGraph& b) {
                                  return a.last_use < b.last_use;
                                });
    cudaGraphExecDestroy(lru->exec);
    model->graphs.erase(lru);
  }
  j1_model::ForwardGraph g;
  std::copy(key.begin(), key.end(), g.key);
  g.exec = exec;
  g.launches = model->launches;
  g.last_use = ++model->graph_tick;
  model->graphs.push_back(g);
  J1_TRY_CUDA(cudaGraphLaunch(exec, model->stream), "forward graph launch");
  return J1_OK;
}

// Waits for a slot's forward and copies its m scores out (checking the error word and
// finiteness, as Engine::forward does with the logits, src/engine.rs:219-221).
j1_status collect(j1_model* model, int slot, float* scores_out, size_t m) {
  J1_TRY_CUDA(cudaEventSynchronize(model->slot_done[slot]), "forward");
  if (model->err_host[slot] != 0) {
    const int code = model->err_host[slot];
    cudaStreamSynchronize(model->stream);
    cudaMemsetAsync(model->err_dev, 0, 4, model->stream);
    cudaStreamSynchronize(model->stream);
    model->err_host[slot] = 0;
    return set_error(J1_ERR_DEVICE_TIMEOUT,
                     "device-side wait timed out (site " + std::to_string(code >> 16) + "); results discarded");
  }
  float* sc = model->scores_host[slot];
  if (m && take_fault(J1_FAULT_NAN)) sc[0] = std::numeric_limits<float>::quiet_NaN();
  for (size_t i = 0; i < m; ++i)
    if (!std::isfinite(sc[i])) return set_error(J1_ERR_NONFINITE, "Inference returned nonfinite logits");
  if (m) std::memcpy(scores_out, sc, m * 4);
  return J1_OK;
}

j1_status finish_forward(j1_model* model, float* scores_out, size_t m) {
  if (!model->staged) return set_error(J1_ERR_INVALID_ARG, "no staged batch");
  if (m != model->m) return set_error(J1_ERR_INVALID_ARG, "scores length does not match the staged batch");
  if (m && !scores_out) return set_error(J1_ERR_INVALID_ARG, "scores_out is NULL");
  j1_status s = enqueue_readback(model);
  if (s) return s;
  s = collect(model, model->slot, scores_out, m);
  prof_fold(model);
  return s;
}

// Several batches back to back: batch k + 1 is validated, packed and uploaded while batch
// k computes (two staging slots); scores are collected one batch behind.
j1_status forward_many(j1_model* model, const std::vector<BatchView>& batches, float* const* outs) {
  size_t T = 0, Mk = 0, E = 0;
  for (size_t k = 0; k < batches.size(); ++k) {
    j1_status s = validate_batch(model, batches[k]);
    if (s) return set_error(s, "batch " + std::to_string(k) + ": " + t_last_error);
    if (batches[k].m && !outs[k]) return set_error(J1_ERR_INVALID_ARG, "scores_out is NULL");
    T = std::max(T, batches[k].t);
    Mk = std::max(Mk, batches[k].m);
    E = std::max(E, meta_layout(batches[k]).ints);
  }
  J1_TRY_CUDA(cudaStreamSynchronize(model->stream), "forward");
  j1_status s = ensure_workspace(model, T, Mk, E);  // no growth (and no reallocation) below
  if (s) return s;
  model->slot_busy[0] = model->slot_busy[1] = false;
  int prev = -1;
  for (size_t k = 0; k < batches.size(); ++k) {
    const int slot = static_cast<int>(k & 1);
    if ((s = stage_batch(model, batches[k], slot, false)) || (s = launch_forward(model)) ||
        (s = enqueue_readback(model)))
      break;
    if (prev >= 0 && (s = collect(model, prev & 1, outs[prev], batches[prev].m))) break;
    prev = static_cast<int>(k);
  }
  if (!s && prev >= 0) s = collect(model, prev & 1, outs[prev], batches[prev].m);
  cudaStreamSynchronize(model->stream);  // nothing of this call stays in flight
  model->slot_busy[0] = model->slot_busy[1] = false;
  prof_fold(model);
  return s;
}

// Every tensor HostWeights::load reads (src/model.rs:55-110), with its shape; checked
// before any device work so a bad checkpoint fails fast (and without a GPU).
j1_status validate_checkpoint(SafeTensors& st, const ModelConfig& c) {
  const size_t H = c.hidden, I = c.intermediate, FF = c.head_ff;
  std::vector<std::pair<std::string, std::vector<size_t>>> want = {
      {"encoder.embeddings.tok_embeddings.weight", {size_t(c.vocab), H}},
      {"encoder.embeddings.norm.weight", {H}},
      {"encoder.final_norm.weight", {H}},
      {"type_emb.weight", {3, H}},
      {"scorer.0.weight", {H}}, {"scorer.0.bias", {H}}, {"scorer.1.weight", {H, H}}, {"scorer.1.bias", {H}},
      {"scorer.3.weight", {1, H}}, {"scorer.3.bias", {1}}};
  for (int l = 0; l < c.layers; ++l) {
    const std::string pre = "encoder.layers." + std::to_string(l) + ".";
    if (l > 0) want.push_back({pre + "attn_norm.weight", {H}});
    want.push_back({pre + "attn.Wqkv.weight", {3 * H, H}});
    want.push_back({pre + "attn.Wo.weight", {H, H}});
    want.push_back({pre + "mlp_norm.weight", {H}});
    want.push_back({pre + "mlp.Wi.weight", {2 * I, H}});
    want.push_back({pre + "mlp.Wo.weight", {H, I}});
  }
  for (int j = 0; j < c.head_layers; ++j) {
    const std::string pre = "head.layers." + std::to_string(j) + ".";
    for (auto& kv : std::vector<std::pair<const char*, std::vector<size_t>>>{
             {"norm1.weight", {H}}, {"norm1.bias", {H}}, {"self_attn.in_proj_weight", {3 * H, H}},
             {"self_attn.in_proj_bias", {3 * H}}, {"self_attn.out_proj.weight", {H, H}},
             {"self_attn.out_proj.bias", {H}}, {"norm2.weight", {H}}, {"norm2.bias", {H}},
             {"linear1.weight", {FF, H}}, {"linear1.bias", {FF}}, {"linear2.weight", {H, FF}},
             {"linear2.bias", {H}}})
      want.push_back({pre + kv.first, kv.second});
  }
  std::string err;
  for (const auto& w : want)
    if (!st.f32(w.first, w.second, err)) return set_error(J1_ERR_IO, err);
  return J1_OK;
}

void destroy_model(j1_model* model);

j1_status create_model(const char* ckpt_dir, int ordinal, j1_model** out) {
  if (!ckpt_dir || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
  *out = nullptr;
  const std::string root(ckpt_dir);
  std::unique_ptr<j1_model, void (*)(j1_model*)> model(new j1_model(), destroy_model);
  std::string err;
  if (!config_load(root, model->cfg, err)) return set_error(J1_ERR_IO, err);
  if (file_exists(root + "/INCOMPLETE") || file_exists(root + "/quantization.json"))
    return set_error(J1_ERR_UNSUPPORTED, "INT8 checkpoints are not supported by this runtime");
  const ModelConfig& c = model->cfg;
  if (!hidden_supported(c.hidden) || c.head_dim != 64)
    return set_error(J1_ERR_UNSUPPORTED,
                     "CUDA kernels are specialized for hidden 256/384/512/768/1024 / head_dim 64");
  if (c.intermediate % 128 != 0) return set_error(J1_ERR_UNSUPPORTED, "intermediate_size must be a multiple of 128");
  if (c.head_heads != c.heads || c.head_layers < 1)
    return set_error(J1_ERR_UNSUPPORTED, "Unsupported decision head layout");
  SafeTensors st;
  if (!st.open(root + "/model.safetensors", err)) return set_error(J1_ERR_IO, err);
  if (j1_status v = validate_checkpoint(st, c)) return v;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return set_error(J1_ERR_CUDA, "CUDA device unavailable");
  if (ordinal < 0 || ordinal >= ndev) return set_error(J1_ERR_CUDA, "CUDA device unavailable");
  DeviceGuard guard(ordinal);
  if (!guard.ok()) return set_error(J1_ERR_CUDA, "CUDA device unavailable");
  model->device = ordinal;
  cudaDeviceProp prop;
  J1_TRY_CUDA(cudaGetDeviceProperties(&prop, ordinal), "device properties");
  if (prop.major != 10 || prop.minor != 0)
    return set_error(J1_ERR_UNSUPPORTED, "this build targets sm_100a (B200); device is sm_" +
                                             std::to_string(prop.major) + std::to_string(prop.minor));
  model->num_sms = prop.multiProcessorCount;
  model->name = "cuda:" + std::to_string(ordinal) + " (" + prop.name + ")";
  J1_TRY_CUDA(cudaStreamCreateWithFlags(&model->stream, cudaStreamNonBlocking), "stream");
  j1_model* M = model.get();
  void* p;
  j1_status s;
  if ((s = dalloc(M, &p, 4, M->allocations))) return s;
  M->err_dev = static_cast<int*>(p);
  J1_TRY_CUDA(cudaMemsetAsync(M->err_dev, 0, 4, M->stream), "memset");
  J1_TRY_CUDA(cudaMallocHost(&p, 16), "cudaMallocHost");
  M->err_host = static_cast<int*>(p);
  std::memset(M->err_host, 0, 16);
  for (int k = 0; k < 2; ++k)
    J1_TRY_CUDA(cudaEventCreateWithFlags(&M->slot_done[k], cudaEventDisableTiming), "event");

  const size_t H = c.hidden, I = c.intermediate, FF = c.head_ff;
  // staging for FP32 -> BF16 conversion, sized for the largest GEMM weight
  const size_t stage_elems = std::max({3 * H * H, 2 * I * H, FF * H});
  if ((s = dalloc(M, &p, stage_elems * 4, M->allocations))) return s;
  float* staging = static_cast<float*>(p);

  if ((s = upload_f32(M, st, "encoder.embeddings.tok_embeddings.weight", {size_t(c.vocab), H}, &M->emb))) return s;
  if ((s = upload_f32(M, st, "encoder.embeddings.norm.weight", {H}, &M->emb_norm))) return s;
  std::vector<float> thetas;
  const int bn_full = gemm_bn_for(static_cast<int>(H)), bn_qkv = gemm_bn_for(static_cast<int>(3 * H));
  const int bn_ff = gemm_bn_for(static_cast<int>(FF));
  for (int l = 0; l < c.layers; ++l) {
    j1_model::Layer ly;
    const std::string pre = "encoder.layers." + std::to_string(l) + ".";
    const float theta = c.rope_theta[l];
    int rope = -1;
    for (size_t k = 0; k < thetas.size(); ++k)
      if (thetas[k] == theta) rope = static_cast<int>(k);
    if (rope < 0) {
      std::vector<float> ct, sn;
      rope_table(theta, c.head_dim, c.max_positions, ct, sn);
      float *dc, *ds;
      if ((s = dalloc(M, &p, ct.size() * 4, M->allocations))) return s;
      dc = static_cast<float*>(p);
      if ((s = dalloc(M, &p, sn.size() * 4, M->allocations))) return s;
      ds = static_cast<float*>(p);
      J1_TRY_CUDA(cudaMemcpyAsync(dc, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice, M->stream), "rope upload");
      J1_TRY_CUDA(cudaMemcpyAsync(ds, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice, M->stream), "rope upload");
      J1_TRY_CUDA(cudaStreamSynchronize(M->stream), "rope upload");
      M->rope_cos.push_back(dc);
      M->rope_sin.push_back(ds);
      thetas.push_back(theta);
      rope = static_cast<int>(thetas.size()) - 1;
    }
    ly.rope = rope;
    ly.global = c.global[l];
    if (l > 0 && (s = upload_f32(M, st, pre + "attn_norm.weight", {H}, &ly.attn_norm))) return s;
    if ((s = upload_f32(M, st, pre + "mlp_norm.weight", {H}, &ly.mlp_norm))) return s;
    if ((s = upload_bf16(M, st, pre + "attn.Wqkv.weight", 3 * H, H, 0, staging, &ly.wqkv, &ly.tm_wqkv, bn_qkv)))
      return s;
    if ((s = upload_bf16(M, st, pre + "attn.Wo.weight", H, H, 0, staging, &ly.wo, &ly.tm_wo, bn_full))) return s;
    if ((s = upload_bf16(M, st, pre + "mlp.Wi.weight", 2 * I, H, static_cast<int>(I), staging, &ly.wi, &ly.tm_wi,
                         256)))
      return s;
    if ((s = upload_bf16(M, st, pre + "mlp.Wo.weight", H, I, 0, staging, &ly.wo2, &ly.tm_wo2, bn_full))) return s;
    M->layers.push_back(ly);
  }
  if ((s = upload_f32(M, st, "encoder.final_norm.weight", {H}, &M->final_norm))) return s;
  if ((s = upload_f32(M, st, "type_emb.weight", {3, H}, &M->type_emb))) return s;
  for (int j = 0; j < c.head_layers; ++j) {
    j1_model::Head hl;
    std::memset(&hl, 0, sizeof(hl));
    const std::string pre = "head.layers." + std::to_string(j) + ".";
    if ((s = upload_f32(M, st, pre + "norm1.weight", {H}, &hl.norm1_w)) ||
        (s = upload_f32(M, st, pre + "norm1.bias", {H}, &hl.norm1_b)) ||
        (s = upload_f32(M, st, pre + "self_attn.in_proj_bias", {3 * H}, &hl.in_b)) ||
        (s = upload_f32(M, st, pre + "self_attn.out_proj.bias", {H}, &hl.out_b)) ||
        (s = upload_f32(M, st, pre + "norm2.weight", {H}, &hl.norm2_w)) ||
        (s = upload_f32(M, st, pre + "norm2.bias", {H}, &hl.norm2_b)) ||
        (s = upload_f32(M, st, pre + "linear1.bias", {FF}, &hl.lin1_b)) ||
        (s = upload_f32(M, st, pre + "linear2.bias", {H}, &hl.lin2_b)) ||
        (s = upload_bf16(M, st, pre + "self_attn.in_proj_weight", 3 * H, H, 0, staging, &hl.in_w, &hl.tm_in, bn_qkv)) ||
        (s = upload_bf16(M, st, pre + "self_attn.out_proj.weight", H, H, 0, staging, &hl.out_w, &hl.tm_out, bn_full)) ||
        (s = upload_bf16(M, st, pre + "linear1.weight", FF, H, 0, staging, &hl.lin1_w, &hl.tm_lin1, bn_ff)) ||
        (s = upload_bf16(M, st, pre + "linear2.weight", H, FF, 0, staging, &hl.lin2_w, &hl.tm_lin2, bn_full)))
      return s;
    const char* why = nullptr;
    if (!make_tmap_bf16(&hl.tm_in_q, hl.in_w, H, H, H, gemm_w_box_rows(bn_full), &why) ||
        !make_tmap_bf16(&hl.tm_in_kv, hl.in_w + static_cast<size_t>(H) * H, 2 * H, H, H,
                        gemm_w_box_rows(gemm_bn_for(static_cast<int>(2 * H))), &why))
      return set_error(J1_ERR_CUDA, std::string("weight tensor map: ") + (why ? why : ""));
    M->head.push_back(hl);
  }
  if ((s = upload_f32(M, st, "scorer.0.weight", {H}, &M->s_norm_w)) ||
      (s = upload_f32(M, st, "scorer.0.bias", {H}, &M->s_norm_b)) ||
      (s = upload_f32(M, st, "scorer.1.bias", {H}, &M->s_b1)) ||
      (s = upload_f32(M, st, "scorer.3.weight", {1, H}, &M->s_w2)) ||
      (s = upload_bf16(M, st, "scorer.1.weight", H, H, 0, staging, &M->s_w1, &M->tm_s_w1, bn_full)))
    return s;
  {
    const float* b2 = st.f32("scorer.3.bias", {1}, err);
    if (!b2) return set_error(J1_ERR_IO, err);
    M->s_b2 = b2[0];
  }
  J1_TRY_CUDA(cudaDeviceSynchronize(), "weight upload");
  *out = model.release();
  return J1_OK;
}

void destroy_model(j1_model* model) {
  if (!model) return;
  DeviceGuard guard(model->device);
  if (model->stream) cudaStreamSynchronize(model->stream);
  free_workspace(model);
  for (cudaEvent_t e : model->prof_ev) cudaEventDestroy(e);
  for (cudaEvent_t e : model->slot_done)
    if (e) cudaEventDestroy(e);
  for (void* p : model->allocations) cudaFree(p);
  if (model->err_host) cudaFreeHost(model->err_host);
  if (model->stream) cudaStreamDestroy(model->stream);
  delete model;
}

// ---------------------------------------------------------------- op-level state (per device)
struct OpState {
  int* err = nullptr;
  int num_sms = 0;
  AttnTile* tiles = nullptr;
  size_t tiles_cap = 0;
};
std::mutex g_op_mu;
std::unordered_map<int, OpState> g_ops;

j1_status op_state(OpState** out) {
  int dev = 0;
  J1_TRY_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  std::lock_guard<std::mutex> lk(g_op_mu);
  OpState& s = g_ops[dev];
  if (!s.err) {
    void* p;
    J1_TRY_CUDA(cudaMalloc(&p, 4), "cudaMalloc");
    J1_TRY_CUDA(cudaMemset(p, 0, 4), "cudaMemset");
    s.err = static_cast<int*>(p);
    J1_TRY_CUDA(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev), "device attribute");
  }
  *out = &s;
  return J1_OK;
}

j1_status op_sync_check(OpState* s, cudaStream_t st) {
  J1_TRY_CUDA(cudaStreamSynchronize(st), "op");
  int e = 0;
  J1_TRY_CUDA(cudaMemcpy(&e, s->err, 4, cudaMemcpyDeviceToHost), "op error word");
  if (e) {
    cudaMemset(s->err, 0, 4);
    return set_error(J1_ERR_DEVICE_TIMEOUT, "device-side wait timed out (site " + std::to_string(e >> 16) + ")");
  }
  return J1_OK;
}

}  // namespace

// ================================================================== C ABI
extern "C" {

size_t j1_last_error(char* buf, size_t cap) { return last_error_copy(buf, cap); }

const char* j1_status_name(j1_status s) {
  switch (s) {
    case J1_OK: return "J1_OK";
    case J1_ERR_INVALID_ARG: return "J1_ERR_INVALID_ARG";
    case J1_ERR_UNSUPPORTED: return "J1_ERR_UNSUPPORTED";
    case J1_ERR_CUDA: return "J1_ERR_CUDA";
    case J1_ERR_OOM: return "J1_ERR_OOM";
    case J1_ERR_NONFINITE: return "J1_ERR_NONFINITE";
    case J1_ERR_DEVICE_TIMEOUT: return "J1_ERR_DEVICE_TIMEOUT";
    case J1_ERR_IO: return "J1_ERR_IO";
    case J1_ERR_INTERNAL: return "J1_ERR_INTERNAL";
  }
  return "J1_ERR_UNKNOWN";
}

const char* j1_version(void) { return "libj1 0.1.0 sm_100a"; }

j1_status j1_config_load(const char* ckpt_dir, j1_config* out) {
  return guard("j1_config_load", [&]() -> j1_status {
    if (!ckpt_dir || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    ModelConfig c;
    std::string err;
    if (!config_load(ckpt_dir, c, err)) return set_error(J1_ERR_IO, err);
    out->hidden = c.hidden;
    out->heads = c.heads;
    out->head_dim = c.head_dim;
    out->intermediate = c.intermediate;
    out->layers = c.layers;
    out->half_window = c.half_window;
    out->vocab = c.vocab;
    out->max_positions = c.max_positions;
    out->head_layers = c.head_layers;
    out->head_heads = c.head_heads;
    out->head_ff = c.head_ff;
    out->norm_eps = c.norm_eps;
    out->n_global = 0;
    for (bool g : c.global) out->n_global += g ? 1 : 0;
    return J1_OK;
  });
}

void j1_inject_fault(int32_t kind, int32_t count) {
  if (kind >= J1_FAULT_ALLOC && kind <= J1_FAULT_DEVICE_WAIT) g_fault[kind] = count > 0 ? count : 0;
}

j1_status j1_selftest_device_timeout(int ordinal, int64_t limit_cycles) {
  return guard("j1_selftest_device_timeout", [&]() -> j1_status {
    int n = 0;
    J1_TRY_CUDA(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
    if (ordinal < 0 || ordinal >= n) return set_error(J1_ERR_INVALID_ARG, "no such device");
    if (limit_cycles < 1000 || limit_cycles > 4000000000LL)
      return set_error(J1_ERR_INVALID_ARG, "limit_cycles must be in [1e3, 4e9]");
    J1_TRY_CUDA(cudaSetDevice(ordinal), "cudaSetDevice");
    int* err = nullptr;
    J1_TRY_CUDA(cudaMalloc(&err, 4), "cudaMalloc");
    int code = 0;
    cudaError_t e = cudaMemset(err, 0, 4);
    if (e == cudaSuccess) e = static_cast<cudaError_t>(launch_wait_timeout_selftest(err, limit_cycles, nullptr));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&code, err, 4, cudaMemcpyDeviceToHost);
    cudaFree(err);
    if (e != cudaSuccess) return cuda_error(e, "device timeout self-test");
    if (code == 0) return set_error(J1_ERR_CUDA, "device timeout self-test: the wait did not time out");
    return set_error(J1_ERR_DEVICE_TIMEOUT,
                     "device-side wait timed out (site " + std::to_string(code >> 16) + "); self-test");
  });
}

j1_status j1_model_create(const char* ckpt_dir, int ordinal, j1_model** out) {
  return guard("j1_model_create", [&]() -> j1_status {
    // J1_FAULT=alloc|launch|nan|host|worker arms one injected fault for the process (j1_inject_fault)
    if (const char* f = std::getenv("J1_FAULT")) {
      static std::atomic<bool> armed{false};
      if (!armed.exchange(true)) {
        const std::string k(f);
        j1_inject_fault(k == "alloc"    ? J1_FAULT_ALLOC
                        : k == "launch" ? J1_FAULT_LAUNCH
                        : k == "nan"    ? J1_FAULT_NAN
                        : k == "host"   ? J1_FAULT_HOST
                        : k == "worker" ? J1_FAULT_WORKER
                                        : 0,
                        1);
      }
    }
    j1_status s = create_model(ckpt_dir, ordinal, out);
    return s;
  });
}

void j1_model_destroy(j1_model* model) { destroy_model(model); }

size_t j1_model_name(const j1_model* model, char* buf, size_t cap) {
  if (!model) {
    if (buf && cap) buf[0] = 0;
    return 0;
  }
  return copy_out(model->name, buf, cap);
}

j1_status j1_model_config(const j1_model* model, j1_config* out) {
  return guard("j1_model_config", [&]() -> j1_status {
    if (!model || !out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    const ModelConfig& c = model->cfg;
    out->hidden = c.hidden;
    out->heads = c.heads;
    out->head_dim = c.head_dim;
    out->intermediate = c.intermediate;
    out->layers = c.layers;
    out->half_window = c.half_window;
    out->vocab = c.vocab;
    out->max_positions = c.max_positions;
    out->head_layers = c.head_layers;
    out->head_heads = c.head_heads;
    out->head_ff = c.head_ff;
    out->norm_eps = c.norm_eps;
    out->n_global = 0;
    for (bool g : c.global) out->n_global += g ? 1 : 0;
    return J1_OK;
  });
}

j1_status j1_model_stage(j1_model* model, const uint32_t* ids, size_t t, const uint32_t* starts,
                         const uint32_t* lens, const uint8_t* qtypes, size_t nseq, const uint32_t* marker_rows,
                         const uint32_t* marker_starts, size_t m) {
  return guard("j1_model_stage", [&]() -> j1_status {
    if (!model) return set_error(J1_ERR_INVALID_ARG, "NULL model");
    std::lock_guard<std::mutex> lk(model->mu);
    DeviceGuard guard(model->device);
    BatchView b{ids, t, starts, lens, qtypes, nseq, marker_rows, marker_starts, m};
    return stage_batch(model, b);
  });
}

j1_status j1_model_launch(j1_model* model) {
  return guard("j1_model_launch", [&]() -> j1_status {
    if (!model) return set_error(J1_ERR_INVALID_ARG, "NULL model");
    std::lock_guard<std::mutex> lk(model->mu);
    DeviceGuard guard(model->device);
    return launch_forward(model);
  });
}

j1_status j1_model_finish(j1_model* model, float* scores_out, size_t m) {
  return guard("j1_model_finish", [&]() -> j1_status {
    if (!model) return set_error(J1_ERR_INVALID_ARG, "NULL model");
    std::lock_guard<std::mutex> lk(model->mu);
    DeviceGuard guard(model->device);
    return finish_forward(model, scores_out, m);
  });
}

j1_status j1_model_forward(j1_model* model, const uint32_t* ids, size_t t, const uint32_t* starts,
                           const uint32_t* lens, const uint8_t* qtypes, size_t nseq, const uint32_t* marker_rows,
                           const uint32_t* marker_starts, size_t m, float* scores_out) {
  return guard("j1_model_forward", [&]() -> j1_status {
    if (!model) return set_error(J1_ERR_INVALID_ARG, "NULL model");
    std::lock_guard<std::mutex> lk(model->mu);
    DeviceGuard guard(model->device);
    BatchView b{ids, t, starts, lens, qtypes, nseq, marker_rows, marker_starts, m};
    j1_status s = stage_batch(model, b);
    if (s) return s;
    if ((s = launch_forward(model))) return s;
    return finish_forward(model, scores_out, m);
  });
}

j1_status j1_model_forward_many(j1_model* model, size_t nbatch, const j1_batch* batches, float* const* scores_out) {
  return guard("j1_model_forward_many", [&]() -> j1_status {
    if (!model) return set_error(J1_ERR_INVALID_ARG, "NULL model");
    if (nbatch && (!batches || !scores_out)) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::lock_guard<std::mutex> lk(model->mu);
    DeviceGuard guard(model->device);
    std::vector<BatchView> v;
    v.reserve(nbatch);
    for (size_t k = 0; k < nbatch; ++k) {
      const j1_batch& b = batches[k];
      v.push_back(BatchView{b.ids, b.t, b.starts, b.lens, b.qtypes, b.nseq, b.marker_rows, b.marker_starts, b.m});
    }
    return forward_many(model, v, scores_out);
  });
}

void* j1_model_stream(j1_model* model) { return model ? static_cast<void*>(model->stream) : nullptr; }

int64_t j1_model_launch_count(const j1_model* model) { return model ? model->launches : 0; }

j1_status j1_model_profile(j1_model* model, int enable) {
  return guard("j1_model_profile", [&]() -> j1_status {
    if (!model) return set_error(J1_ERR_INVALID_ARG, "NULL model");
    std::lock_guard<std::mutex> lk(model->mu);
    DeviceGuard guard(model->device);
    J1_TRY_CUDA(cudaStreamSynchronize(model->stream), "profile");
    prof_fold(model);
    model->prof_on = enable != 0;
    for (int i = 0; i < J1_PROF_FAMILIES; ++i) model->prof_ms[i] = 0.0, model->prof_cnt[i] = 0;
    return J1_OK;
  });
}

j1_status j1_model_profile_read(j1_model* model, double* ms, int64_t* launches) {
  return guard("j1_model_profile_read", [&]() -> j1_status {
    if (!model || !ms || !launches) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::lock_guard<std::mutex> lk(model->mu);
    for (int i = 0; i < J1_PROF_FAMILIES; ++i) ms[i] = model->prof_ms[i], launches[i] = model->prof_cnt[i];
    return J1_OK;
  });
}

const char* j1_profile_family_name(int family) {
  return (family >= 0 && family < J1_PROF_FAMILIES) ? kFamilyNames[family] : "";
}

j1_status j1_op_gemm(const j1_gemm_args* a, void* stream, int sync) {
  return guard("j1_op_gemm", [&]() -> j1_status {
    if (!a || !a->A || !a->W) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    const GemmEpi epi = static_cast<GemmEpi>(a->epilogue);
    if (a->epilogue < 0 || a->epilogue > 5) return set_error(J1_ERR_INVALID_ARG, "unknown epilogue");
    const int bn = (epi == EPI_GEGLU) ? 256 : gemm_bn_for(a->N);
    if (const char* why = gemm_shape_error(epi, bn, a->M, a->N, a->K)) return set_error(J1_ERR_UNSUPPORTED, why);
    const bool full_row = epi == EPI_RESID_LN || epi == EPI_RESID || epi == EPI_SCORER;
    if (full_row && a->M > 0 && epi != EPI_SCORER && (a->ldx < a->N || a->ldx % 4 != 0))
      return set_error(J1_ERR_INVALID_ARG, "ldx must be >= N and a multiple of 4");
    if ((epi == EPI_BF16 || epi == EPI_QKV_ROPE || epi == EPI_GEGLU) && !a->out)
      return set_error(J1_ERR_INVALID_ARG, "out is NULL");
    if ((epi == EPI_RESID_LN || epi == EPI_RESID) && !a->x) return set_error(J1_ERR_INVALID_ARG, "x is NULL");
    if (epi == EPI_RESID_LN && (!a->ln_w || !a->xn)) return set_error(J1_ERR_INVALID_ARG, "ln_w/xn is NULL");
    if (epi == EPI_QKV_ROPE && (!a->pos || !a->rope_cos || !a->rope_sin))
      return set_error(J1_ERR_INVALID_ARG, "RoPE tables are NULL");
    if (epi == EPI_SCORER && (!a->bias || !a->w2 || !a->scores)) return set_error(J1_ERR_INVALID_ARG, "scorer args NULL");
    OpState* os;
    j1_status s = op_state(&os);
    if (s) return s;
    CUtensorMap tmA, tmW, tmX;
    const char* why = nullptr;
    if (!make_tmap_bf16(&tmA, a->A, a->M, a->K, a->K, 128, &why) ||
        !make_tmap_bf16(&tmW, a->W, a->N, a->K, a->K, gemm_w_box_rows(bn), &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    const bool resid = epi == EPI_RESID_LN || epi == EPI_RESID;
    if (resid && !make_tmap_f32_resid(&tmX, a->x, a->M, a->N, a->ldx, &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    const bool tile_out = epi == EPI_BF16 || epi == EPI_QKV_ROPE || epi == EPI_GEGLU;
    const int out_cols = epi == EPI_GEGLU ? a->N / 2 : a->N;
    if (tile_out && (a->ldo < out_cols || a->ldo % 8 != 0))
      return set_error(J1_ERR_INVALID_ARG, "ldo must be >= the output width and a multiple of 8");
    if (tile_out && !make_tmap_bf16(&tmX, a->out, a->M, out_cols, a->ldo, 128, &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    CUtensorMap tmXN, tmXs;
    if (epi == EPI_RESID_LN && (a->ldxn < a->N || a->ldxn % 8 != 0))
      return set_error(J1_ERR_INVALID_ARG, "ldxn must be >= N and a multiple of 8");
    if (epi == EPI_RESID_LN && !make_tmap_bf16(&tmXN, a->xn, a->M, a->N, a->ldxn, 32, &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    if (resid && !make_tmap_f32_resid(&tmXs, a->x, a->M, a->N, a->ldx, &why, 32))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    EpiParams p;
    std::memset(&p, 0, sizeof(p));
    p.M = a->M, p.N = a->N, p.K = a->K;
    p.out = static_cast<bf16*>(a->out), p.ldo = a->ldo;
    p.bias = a->bias, p.relu = a->relu;
    p.x = a->x, p.ldx = a->ldx;
    p.ln_w = a->ln_w, p.ln_b = a->ln_b, p.ln_eps = a->ln_eps;
    p.xn = static_cast<bf16*>(a->xn), p.ldxn = a->ldxn;
    p.pos = a->pos, p.rope_cos = a->rope_cos, p.rope_sin = a->rope_sin, p.rope_cols = a->rope_cols;
    p.w2 = a->w2, p.b2 = a->b2, p.scores = a->scores;
    p.err = os->err;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int grid = a->grid_limit > 0 ? a->grid_limit : os->num_sms;
    int rc = launch_gemm(epi, bn, tmA, tmW, (resid || tile_out) ? &tmX : nullptr, p, grid, st,
                         resid ? &tmXs : nullptr, epi == EPI_RESID_LN ? &tmXN : nullptr);
    if (rc) return cuda_error(static_cast<cudaError_t>(rc), "gemm launch");
    return sync ? op_sync_check(os, st) : J1_OK;
  });
}

j1_status j1_op_attention(const void* qkv, int64_t t, int32_t hidden, const uint32_t* seq_starts,
                          const uint32_t* seq_lens, size_t nseq, int32_t window, void* ctx, void* stream, int sync) {
  return guard("j1_op_attention", [&]() -> j1_status {
    if (!qkv || !ctx || (nseq && (!seq_starts || !seq_lens))) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (hidden % 64 != 0 || hidden <= 0) return set_error(J1_ERR_UNSUPPORTED, "hidden must be a multiple of 64");
    std::vector<AttnTile> tiles;
    for (size_t s = 0; s < nseq; ++s) {
      if (seq_lens[s] == 0 || static_cast<int64_t>(seq_starts[s]) + seq_lens[s] > t)
        return set_error(J1_ERR_INVALID_ARG, "sequence outside the qkv buffer");
      const uint32_t PQ = static_cast<uint32_t>(attention_pair_queries());
      for (uint32_t q0 = 0; q0 < seq_lens[s]; q0 += PQ) {
        AttnTile tl;
        tl.q_row0 = static_cast<int>(seq_starts[s] + q0);
        tl.nq = static_cast<int>(std::min<uint32_t>(PQ, seq_lens[s] - q0));
        tl.kv_row0 = static_cast<int>(seq_starts[s]);
        tl.kv_len = static_cast<int>(seq_lens[s]);
        tl.q_pos0 = static_cast<int>(q0);
        tl.pad0 = tl.pad1 = tl.pad2 = 0;
        tiles.push_back(tl);
      }
    }
    OpState* os;
    j1_status s = op_state(&os);
    if (s) return s;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (tiles.size() > os->tiles_cap) {
      J1_TRY_CUDA(cudaDeviceSynchronize(), "op attention");
      if (os->tiles) cudaFree(os->tiles);
      os->tiles = nullptr;
      void* p;
      J1_TRY_CUDA(cudaMalloc(&p, tiles.size() * sizeof(AttnTile)), "cudaMalloc");
      os->tiles = static_cast<AttnTile*>(p);
      os->tiles_cap = tiles.size();
    }
    if (!tiles.empty())
      J1_TRY_CUDA(cudaMemcpyAsync(os->tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, st),
                  "tiles upload");
    CUtensorMap tm;
    const char* why = nullptr;
    if (!make_tmap_bf16(&tm, qkv, static_cast<uint64_t>(t), 3 * static_cast<uint64_t>(hidden), 3 * hidden, 128, &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    CUtensorMap tmO, tmKV;
    if (!make_tmap_bf16(&tmO, ctx, static_cast<uint64_t>(t), static_cast<uint64_t>(hidden), hidden, 32, &why) ||
        !make_tmap_bf16(&tmKV, qkv, static_cast<uint64_t>(t), 3 * static_cast<uint64_t>(hidden), 3 * hidden,
                        attention_kv_box_rows(), &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    int rc = launch_attention(tm, tmKV, &tmO, os->tiles, static_cast<int>(tiles.size()), hidden / 64, 0, hidden, 2 * hidden,
                              static_cast<bf16*>(ctx), hidden, window, kScaleLog2, os->err, os->num_sms, st);
    if (rc) return cuda_error(static_cast<cudaError_t>(rc), "attention launch");
    if (sync || !tiles.empty()) return op_sync_check(os, st);  // tiles are host-owned: wait before returning
    return J1_OK;
  });
}

j1_status j1_op_geglu_interleave(const float* src_dev, void* dst_dev, int32_t inter, int32_t k, void* stream) {
  return guard("j1_op_geglu_interleave", [&]() -> j1_status {
    if (!src_dev || !dst_dev) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (inter % 128 != 0) return set_error(J1_ERR_UNSUPPORTED, "inter must be a multiple of 128");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = launch_f32_to_bf16(src_dev, static_cast<bf16*>(dst_dev), 2LL * inter, k, inter, st);
    if (rc) return cuda_error(static_cast<cudaError_t>(rc), "interleave");
    J1_TRY_CUDA(cudaStreamSynchronize(st), "interleave");
    return J1_OK;
  });
}

}  // extern "C"
