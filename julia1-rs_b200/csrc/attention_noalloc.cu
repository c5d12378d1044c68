// j1_op_attention_noalloc: the varlen attention op of j1_op_attention, with its
// scratch (the 128-query tile list and the device-side error words) in a fixed
// file-scope device array instead of memory allocated at run time.
//
// Who needs it: a caller whose process has handed all free HBM to its own memory
// pool (a serving process whose caching allocator reserves the device up front)
// gets cudaMalloc failures from j1_op_attention's lazily grown tile buffer, and a
// latency-critical loop cannot afford cudaMalloc/cudaFree, which synchronise the
// whole device. This entry point makes no device or pinned allocation at all.
//
// Limits and sharing:
//  * at most kMaxTiles tiles per call (sum over sequences of ceil(len / 128));
//    larger calls are rejected with J1_ERR_INVALID_ARG before anything runs;
//  * every call on a device uses the same array, and every call in the process the
//    same host staging buffer (kMaxTiles tiles, one upload per call). The host side
//    of a call (staging, upload, launch) is serialised by a mutex; on the device,
//    calls issued on one stream are ordered, while calls that overlap there (two
//    streams without an ordering between them) race on the array and give wrong
//    results;
//  * the array is placed in device memory when the module is first used on a device
//    (CUDA loads modules lazily), i.e. by the first call on that device, which also
//    does the set-up (symbol address, SM count) with that device current. A caller
//    whose pool reserves device memory up front makes that first call before the
//    reservation (a call with nseq = 0 does only the set-up); it also belongs before
//    any stream capture.
//
// Device-side timeouts: error word 0 belongs to the kernel of the current call and is
// zero when it starts; word 1 keeps timeouts of earlier calls that nobody has read.
// Each call first runs a one-thread kernel that moves a non-zero word 0 (left by an
// earlier call made with sync = 0, whose status was returned before its kernel ran)
// into word 1 and clears word 0. A call made with sync = 1 waits for its stream, reads
// both words and reports J1_ERR_DEVICE_TIMEOUT for either (the message says which),
// clearing them. So a timeout of a sync = 0 call is reported by the next call on that
// device made with sync = 1; a call with nseq = 0 and sync = 1 only collects.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "model.h"

using namespace j1rt;

namespace {

constexpr int kMaxTiles = 8192;              // 8192 x 32 B = 256 KiB of tile list
constexpr size_t kTilesOffset = 256;         // error words at bytes 0 and 4, tiles from byte 256
constexpr size_t kScratchBytes = kTilesOffset + kMaxTiles * sizeof(AttnTile);
constexpr int kMaxDevices = 64;
constexpr float kScaleLog2 = 0.125f * 1.44269504088896340736f;  // 1/sqrt(64) * log2(e)
constexpr long long kInjectedWaitCycles = 2000000;  // J1_FAULT_DEVICE_WAIT: ~1 ms bounded wait

static_assert(sizeof(AttnTile) == 32, "tile layout");

#define NA_TRY(expr, what)                               \
  do {                                                   \
    cudaError_t e_ = (expr);                             \
    if (e_ != cudaSuccess) return cuda_error(e_, what);  \
  } while (0)

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

// Word 0 (the current kernel's) -> word 1 (pending, first timeout kept); word 0 cleared.
__global__ void fold_error_words(int* w) {
  const int e = w[0];
  if (e != 0) {
    if (w[1] == 0) w[1] = e;
    w[0] = 0;
  }
}

struct DeviceSetup {
  std::once_flag once;
  cudaError_t rc = cudaSuccess;
  unsigned char* scratch = nullptr;
  int num_sms = 0;
};
DeviceSetup g_setup[kMaxDevices];

// Host staging of one call's tile list (one upload per call); guarded by g_host_mutex.
std::mutex g_host_mutex;
AttnTile g_host_tiles[kMaxTiles];

j1_status setup_device(DeviceSetup** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(J1_ERR_UNSUPPORTED, "device ordinal above 63");
  DeviceSetup& s = g_setup[dev];
  std::call_once(s.once, [&s, dev] {
    void* p = nullptr;
    s.rc = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (s.rc == cudaSuccess) s.rc = cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (s.rc == cudaSuccess) s.scratch = static_cast<unsigned char*>(p);
  });
  if (s.rc != cudaSuccess || !s.scratch) return cuda_error(s.rc, "scratch set-up (cudaGetSymbolAddress)");
  *out = &s;
  return J1_OK;
}

}  // namespace

extern "C" j1_status j1_op_attention_noalloc(const void* qkv, int64_t t, int32_t hidden, const uint32_t* seq_starts,
                                             const uint32_t* seq_lens, size_t nseq, int32_t window, void* ctx,
                                             void* stream, int sync) {
  return guard("j1_op_attention_noalloc", [&]() -> j1_status {
    if (!qkv || !ctx || (nseq && (!seq_starts || !seq_lens))) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (hidden % 64 != 0 || hidden <= 0) return set_error(J1_ERR_UNSUPPORTED, "hidden must be a multiple of 64");
    const uint32_t PQ = static_cast<uint32_t>(attention_pair_queries());
    uint64_t ntiles = 0;
    for (size_t s = 0; s < nseq; ++s) {
      if (seq_lens[s] == 0 || static_cast<int64_t>(seq_starts[s]) + seq_lens[s] > t)
        return set_error(J1_ERR_INVALID_ARG, "sequence outside the qkv buffer");
      ntiles += (seq_lens[s] + PQ - 1) / PQ;
    }
    if (ntiles > static_cast<uint64_t>(kMaxTiles))
      return set_error(J1_ERR_INVALID_ARG, "j1_op_attention_noalloc: " + std::to_string(ntiles) +
                                               " query tiles exceed the fixed scratch of " + std::to_string(kMaxTiles) +
                                               " (128 queries per tile); split the call");
    CUtensorMap tm, tmO, tmKV;
    if (ntiles) {
      const char* why = nullptr;
      if (!make_tmap_bf16(&tm, qkv, static_cast<uint64_t>(t), 3 * static_cast<uint64_t>(hidden), 3 * hidden, 128,
                          &why) ||
          !make_tmap_bf16(&tmO, ctx, static_cast<uint64_t>(t), static_cast<uint64_t>(hidden), hidden, 32, &why) ||
          !make_tmap_bf16(&tmKV, qkv, static_cast<uint64_t>(t), 3 * static_cast<uint64_t>(hidden), 3 * hidden,
                          attention_kv_box_rows(), &why))
        return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    }
    DeviceSetup* ds = nullptr;
    j1_status st = setup_device(&ds);
    if (st) return st;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    int* err = reinterpret_cast<int*>(ds->scratch);
    AttnTile* tiles = reinterpret_cast<AttnTile*>(ds->scratch + kTilesOffset);
    {
      std::lock_guard<std::mutex> lock(g_host_mutex);
      // A pageable-source cudaMemcpyAsync returns once the source has been consumed, so
      // the staging buffer is free again when the lock is released; stream order puts the
      // list in place before the kernel below starts.
      size_t n = 0;
      for (size_t s = 0; s < nseq; ++s)
        for (uint32_t q0 = 0; q0 < seq_lens[s]; q0 += PQ) {
          AttnTile& tl = g_host_tiles[n++];
          tl.q_row0 = static_cast<int>(seq_starts[s] + q0);
          tl.nq = static_cast<int>(std::min<uint32_t>(PQ, seq_lens[s] - q0));
          tl.kv_row0 = static_cast<int>(seq_starts[s]);
          tl.kv_len = static_cast<int>(seq_lens[s]);
          tl.q_pos0 = static_cast<int>(q0);
          tl.pad0 = tl.pad1 = tl.pad2 = 0;
        }
      if (n) NA_TRY(cudaMemcpyAsync(tiles, g_host_tiles, n * sizeof(AttnTile), cudaMemcpyHostToDevice, cs),
                    "tile upload");
      fold_error_words<<<1, 1, 0, cs>>>(err);
      NA_TRY(cudaGetLastError(), "error word fold");
      if (ntiles) {
        const int rc = launch_attention(tm, tmKV, &tmO, tiles, static_cast<int>(ntiles), hidden / 64, 0, hidden,
                                        2 * hidden, static_cast<bf16*>(ctx), hidden, window, kScaleLog2, err,
                                        ds->num_sms, cs);
        if (rc) return cuda_error(static_cast<cudaError_t>(rc), "attention launch");
        // injected fault (tests): a bounded wait that times out records its site in word 0,
        // as a timed-out wait of the attention kernel would
        if (take_fault(J1_FAULT_DEVICE_WAIT)) {
          const int r2 = launch_wait_timeout_selftest(err, kInjectedWaitCycles, cs);
          if (r2) return cuda_error(static_cast<cudaError_t>(r2), "injected device wait");
        }
      }
    }
    if (!sync) return J1_OK;
    NA_TRY(cudaStreamSynchronize(cs), "attention");
    int e[2] = {0, 0};
    NA_TRY(cudaMemcpy(e, err, sizeof(e), cudaMemcpyDeviceToHost), "error words");
    if (e[0] == 0 && e[1] == 0) return J1_OK;
    const int zero[2] = {0, 0};
    NA_TRY(cudaMemcpy(err, zero, sizeof(zero), cudaMemcpyHostToDevice), "clear error words");
    std::string msg;
    if (e[0] != 0) msg = "device-side wait timed out (site " + std::to_string(e[0] >> 16) + ")";
    if (e[1] != 0)
      msg += std::string(msg.empty() ? "" : "; ") + "device-side wait timed out in an earlier call made with sync = 0 (site " +
             std::to_string(e[1] >> 16) + ")";
    return set_error(J1_ERR_DEVICE_TIMEOUT, msg);
  });
}
