// Internal model / status helpers shared by model.cpp and engine.cpp.
#pragma once
#include <cuda_runtime.h>

#include <array>
#include <atomic>
#include <exception>
#include <functional>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/j1.h"
#include "checkpoint.h"
#include "kernels.h"

namespace j1rt {

j1_status set_error(j1_status s, const std::string& msg);
// set_error for exception handlers: builds "<fn>: <what>" and never throws.
j1_status set_error_noexcept(j1_status s, const char* fn, const char* what) noexcept;
j1_status cuda_error(cudaError_t e, const char* what);
// j1_inject_fault state: remaining injected faults per kind (J1_FAULT_*).
extern std::atomic<int> g_fault[8];
bool take_fault(int kind);
bool fault_pending(int kind);  // an injected fault of this kind is waiting to be taken

// Every C entry point runs its body through guard(): a C++ exception (host memory
// exhausted, a thread that could not start, ...) becomes a status and a message instead
// of unwinding into the caller's frames, which a C, Rust or ctypes caller cannot survive.
template <class F>
j1_status guard(const char* fn, F&& body) noexcept {
  try {
    if (take_fault(J1_FAULT_HOST)) throw std::bad_alloc();
    return body();
  } catch (const std::bad_alloc&) {
    return set_error_noexcept(J1_ERR_OOM, fn, "host memory exhausted");
  } catch (const std::exception& e) {
    return set_error_noexcept(J1_ERR_INTERNAL, fn, e.what());
  } catch (...) {
    return set_error_noexcept(J1_ERR_INTERNAL, fn, "unknown C++ exception");
  }
}

// Runs work() on the calling thread and on up to n - 1 more threads. work() takes its
// items from a shared counter, so any number of threads finishes all of them: a thread
// that cannot be started is skipped. An exception inside work() on any thread is caught
// there and rethrown here (the first one) once every started thread has been joined.
void run_pool(int n, const std::function<void()>& work);

// Rows per chunk when j1_engine_logits_text overlaps text encoding with the forward: four
// of the engine's micro-batches per device (at least 256 rows).
size_t engine_pipeline_rows(const j1_engine* e);

// Restores the calling thread's current device on scope exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
    ok_ = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev_ >= 0) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = -1;
  bool ok_ = false;
};

// A packed batch (model::Batch, src/model.rs:225-269) as host views.
struct BatchView {
  const uint32_t* ids;
  size_t t;
  const uint32_t* starts;
  const uint32_t* lens;
  const uint8_t* qtypes;
  size_t nseq;
  const uint32_t* marker_rows;
  const uint32_t* marker_starts;
  size_t m;
};

}  // namespace j1rt

struct j1_model {
  j1rt::ModelConfig cfg;
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  std::string name;
  std::mutex mu;
  std::vector<void*> allocations;  // device memory owned by the model

  // ---- weights (device)
  float* emb = nullptr;
  float* emb_norm = nullptr;
  struct Layer {
    float* attn_norm = nullptr;  // nullptr at layer 0 (nn.Identity)
    float* mlp_norm = nullptr;
    j1rt::bf16 *wqkv = nullptr, *wo = nullptr, *wi = nullptr, *wo2 = nullptr;  // wi interleaved for GEGLU
    CUtensorMap tm_wqkv, tm_wo, tm_wi, tm_wo2;
    int rope = 0;
    bool global = false;
  };
  std::vector<Layer> layers;
  float* final_norm = nullptr;
  float* type_emb = nullptr;
  struct Head {
    float *norm1_w, *norm1_b, *in_b, *out_b, *norm2_w, *norm2_b, *lin1_b, *lin2_b;
    j1rt::bf16 *in_w, *out_w, *lin1_w, *lin2_w;
    CUtensorMap tm_in, tm_out, tm_lin1, tm_lin2;
    CUtensorMap tm_in_q, tm_in_kv;  // in_proj rows [0, H) (queries) and [H, 3H) (keys, values)
  };
  std::vector<Head> head;
  float *s_norm_w = nullptr, *s_norm_b = nullptr, *s_b1 = nullptr, *s_w2 = nullptr;
  float s_b2 = 0.f;
  j1rt::bf16* s_w1 = nullptr;
  CUtensorMap tm_s_w1;
  std::vector<float*> rope_cos, rope_sin;
  int* err_dev = nullptr;

  // ---- workspace (grows monotonically, like ensure_workspace in src/cuda/mod.rs:282-332)
  size_t cap_tokens = 0, cap_markers = 0, cap_meta = 0;
  float* x = nullptr;
  j1rt::bf16 *xn = nullptr, *qkv = nullptr, *ctx = nullptr, *g = nullptr;
  float* ym = nullptr;
  j1rt::bf16 *ymb = nullptr, *cm = nullptr, *hm = nullptr, *qm = nullptr;
  float* scores = nullptr;
  // Two staging slots (batch metadata in/out), so that the next batch can be packed and
  // uploaded while the current one computes (j1_model_forward_many); the single-batch
  // calls use slot 0. err_host holds one error word per slot.
  int* meta_dev[2] = {nullptr, nullptr};
  int* meta_host[2] = {nullptr, nullptr};      // pinned
  float* scores_host[2] = {nullptr, nullptr};  // pinned
  cudaEvent_t slot_done[2] = {nullptr, nullptr};  // the slot's forward and readback completed
  bool slot_busy[2] = {false, false};
  int* err_host = nullptr;  // pinned
  std::vector<void*> ws_allocations;

  // ---- staged batch
  bool staged = false;
  int slot = 0;  // staging slot of the staged batch
  size_t t = 0, m = 0, nseq = 0, ntiles = 0, nmtiles = 0;
  int *d_ids = nullptr, *d_pos = nullptr, *d_qtype = nullptr, *d_markers = nullptr;
  j1rt::AttnTile* d_tiles = nullptr;
  j1rt::AttnTile* d_mtiles = nullptr;  // marker-query tiles of the last head layer
  CUtensorMap tm_xn, tm_ctx, tm_g, tm_h, tm_qkv, tm_cm, tm_ymb, tm_hm;
  CUtensorMap tm_qm, tm_qkv_kv;  // marker queries [m, H]; the k|v columns of qkv
  CUtensorMap tm_ctx_o, tm_cm_o;  // attention outputs, 64 x 32 boxes (TMA stores of O)
  CUtensorMap tm_kv;              // qkv with K/V-block boxes for attention
  CUtensorMap tm_x, tm_ym;  // FP32 residual streams (tokens, markers)
  CUtensorMap tm_x_st, tm_ym_st;    // the same with 32-row boxes (per-warp stores of the residual GEMMs)
  CUtensorMap tm_xn_st, tm_ymb_st;  // LayerNorm outputs with 64 x 32 boxes (per-warp stores)
  int64_t launches = 0;

  // ---- CUDA graphs of the forward's launch sequence, one per batch shape (t, m, nseq,
  // query tiles, marker tiles, staging slot, workspace generation): every kernel argument
  // (pointers, tensor maps, grids) is a function of that key, the batch's contents live in
  // device buffers. A shape is captured the second time it is launched and replayed from
  // then on; J1_GRAPH=0 disables this.
  struct ForwardGraph {
    uint64_t key[7];
    cudaGraphExec_t exec;
    int64_t launches;  // kernels in the graph
    uint64_t last_use;
  };
  std::vector<ForwardGraph> graphs;                 // the least recently used is evicted beyond 8
  std::vector<std::array<uint64_t, 7>> shapes_seen;  // keys launched once and not captured (at most 16)
  uint64_t ws_gen = 0;                              // bumped whenever the workspace is freed
  uint64_t graph_tick = 0;

  // ---- optional per-launch CUDA-event timing by kernel family (j1_model_profile)
  bool prof_on = false;
  std::vector<cudaEvent_t> prof_ev;     // pool: 2 per recorded launch
  std::vector<int> prof_fam;            // family of each recorded launch
  size_t prof_used = 0;                 // recorded launches not yet accumulated
  double prof_ms[J1_PROF_FAMILIES] = {0};
  int64_t prof_cnt[J1_PROF_FAMILIES] = {0};
};
