// j1_op_attention_noalloc: the varlen attention op of j1_op_attention, with its
// scratch (the 128-query tile list and the device-side error word) in a fixed
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
//  * every call on a device uses the same array: the error word must be zero when
//    a call's kernel starts (each call clears it on its stream before the launch),
//    and the tile list is rewritten by each call. Calls issued on one stream are
//    ordered; calls that overlap (two host threads, or two streams without an
//    ordering between them) race on the array and give wrong results;
//  * the first call on each device does the set-up (symbol address, SM count) with
//    that device current; it should happen before any stream capture is begun.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "model.h"

using namespace j1rt;

namespace {

constexpr int kMaxTiles = 8192;              // 8192 x 32 B = 256 KiB of tile list
constexpr size_t kTilesOffset = 256;         // error word at byte 0, tiles from byte 256
constexpr size_t kScratchBytes = kTilesOffset + kMaxTiles * sizeof(AttnTile);
constexpr int kMaxDevices = 64;
constexpr int kChunk = 64;                   // tiles staged on the host stack per copy
constexpr float kScaleLog2 = 0.125f * 1.44269504088896340736f;  // 1/sqrt(64) * log2(e)

static_assert(sizeof(AttnTile) == 32, "tile layout");

#define NA_TRY(expr, what)                               \
  do {                                                   \
    cudaError_t e_ = (expr);                             \
    if (e_ != cudaSuccess) return cuda_error(e_, what);  \
  } while (0)

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

struct DeviceSetup {
  std::once_flag once;
  cudaError_t rc = cudaSuccess;
  unsigned char* scratch = nullptr;
  int num_sms = 0;
};
DeviceSetup g_setup[kMaxDevices];

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
    CUtensorMap tm;
    const char* why = nullptr;
    if (!make_tmap_bf16(&tm, qkv, static_cast<uint64_t>(t), 3 * static_cast<uint64_t>(hidden), 3 * hidden, 128, &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    CUtensorMap tmO, tmKV;
    if (!make_tmap_bf16(&tmO, ctx, static_cast<uint64_t>(t), static_cast<uint64_t>(hidden), hidden, 32, &why) ||
        !make_tmap_bf16(&tmKV, qkv, static_cast<uint64_t>(t), 3 * static_cast<uint64_t>(hidden), 3 * hidden,
                        attention_kv_box_rows(), &why))
      return set_error(J1_ERR_INVALID_ARG, std::string("tensor map: ") + (why ? why : ""));
    DeviceSetup* ds = nullptr;
    j1_status st = setup_device(&ds);
    if (st) return st;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    int* err = reinterpret_cast<int*>(ds->scratch);
    AttnTile* tiles = reinterpret_cast<AttnTile*>(ds->scratch + kTilesOffset);

    // The tile list goes up in stack-sized chunks. A pageable-source cudaMemcpyAsync
    // returns once the source has been consumed, so the chunk can be refilled at once;
    // stream order puts every chunk in place before the kernel below starts.
    AttnTile chunk[kChunk];
    int fill = 0;
    size_t done = 0;
    for (size_t s = 0; s < nseq; ++s)
      for (uint32_t q0 = 0; q0 < seq_lens[s]; q0 += PQ) {
        AttnTile& tl = chunk[fill++];
        tl.q_row0 = static_cast<int>(seq_starts[s] + q0);
        tl.nq = static_cast<int>(std::min<uint32_t>(PQ, seq_lens[s] - q0));
        tl.kv_row0 = static_cast<int>(seq_starts[s]);
        tl.kv_len = static_cast<int>(seq_lens[s]);
        tl.q_pos0 = static_cast<int>(q0);
        tl.pad0 = tl.pad1 = tl.pad2 = 0;
        if (fill == kChunk) {
          NA_TRY(cudaMemcpyAsync(tiles + done, chunk, sizeof(chunk), cudaMemcpyHostToDevice, cs), "tile upload");
          done += kChunk;
          fill = 0;
        }
      }
    if (fill)
      NA_TRY(cudaMemcpyAsync(tiles + done, chunk, fill * sizeof(AttnTile), cudaMemcpyHostToDevice, cs),
                  "tile upload");
    NA_TRY(cudaMemsetAsync(err, 0, sizeof(int), cs), "clear error word");
    const int rc = launch_attention(tm, tmKV, &tmO, tiles, static_cast<int>(ntiles), hidden / 64, 0, hidden, 2 * hidden,
                                    static_cast<bf16*>(ctx), hidden, window, kScaleLog2, err, ds->num_sms, cs);
    if (rc) return cuda_error(static_cast<cudaError_t>(rc), "attention launch");
    if (!sync) return J1_OK;
    NA_TRY(cudaStreamSynchronize(cs), "attention");
    int e = 0;
    NA_TRY(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost), "error word");
    if (e) return set_error(J1_ERR_DEVICE_TIMEOUT, "device-side wait timed out (site " + std::to_string(e >> 16) + ")");
    return J1_OK;
  });
}
