/* libj1: B200-native (sm_100a) encoder forward for Julia-1 / ModernBERT decision models.
 *
 * C ABI replacing the reference's CUDA backend seam (julia1-rs):
 *   enum Backend { Cpu(..), Cuda(Box<CudaModel>) }      src/engine.rs:67-71
 *   CudaModel::new(cfg, &HostWeights, ordinal)           src/cuda/mod.rs:174
 *   CudaModel::forward(&Batch) -> Vec<Vec<f32>>          src/cuda/mod.rs:400
 *   CudaModel::name()                                    src/cuda/mod.rs:278
 *   Engine::logits_encoded / batches / forward           src/engine.rs:191-235
 *
 * Plain pointers and sizes only. The caller owns every host array; the library
 * owns device memory and pinned staging. Every call returns a j1_status and
 * never aborts; j1_last_error() gives the calling thread's last message.
 */
#ifndef J1_H
#define J1_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define J1_API __attribute__((visibility("default")))
#else
#define J1_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* anyhow::Result errors of the reference, as codes. */
typedef enum j1_status {
  J1_OK = 0,
  J1_ERR_INVALID_ARG = 1,       /* bad batch / argument (e.g. marker outside its sequence) */
  J1_ERR_UNSUPPORTED = 2,       /* config the kernels do not support (cf. src/cuda/mod.rs:175-176) */
  J1_ERR_CUDA = 3,              /* CUDA runtime / driver failure; no usable device */
  J1_ERR_OOM = 4,               /* device or pinned allocation failed */
  J1_ERR_NONFINITE = 5,         /* "Inference returned nonfinite logits" (src/engine.rs:219-221) */
  J1_ERR_DEVICE_TIMEOUT = 6,    /* a bounded device-side wait gave up; context still usable */
  J1_ERR_IO = 7,                /* checkpoint / config could not be read or parsed (src/config.rs, src/weights.rs) */
  J1_ERR_INTERNAL = 8           /* a host-side failure inside the library (e.g. a thread that could not start);
                                   host memory exhaustion is J1_ERR_OOM. No C++ exception leaves the library. */
} j1_status;

typedef struct j1_model j1_model;   /* one device replica: CudaModel */
typedef struct j1_engine j1_engine; /* Engine over one or more replicas */

/* Thread-local message of the last failing call on this thread; returns the full length. */
J1_API size_t j1_last_error(char* buf, size_t cap);
J1_API const char* j1_status_name(j1_status s);
/* Library version string, e.g. "libj1 0.1.0 sm_100a". */
J1_API const char* j1_version(void);

/* ------------------------------------------------------------ configuration */
/* ModelConfig (src/config.rs:6-24) as parsed from julia_config.json + encoder/config.json. */
typedef struct j1_config {
  int32_t hidden, heads, head_dim, intermediate, layers;
  int32_t half_window;           /* local_attention / 2 */
  int32_t vocab, max_positions;
  int32_t head_layers, head_heads, head_ff;
  float norm_eps;
  int32_t n_global;              /* layers with i % global_attn_every_n_layers == 0 */
} j1_config;

/* ModelConfig::load (src/config.rs:36-40) without touching a GPU. */
J1_API j1_status j1_config_load(const char* ckpt_dir, j1_config* out);

/* ------------------------------------------------------------ model (one GPU) */
/* CudaModel::new: parses both configs, memory-maps model.safetensors (F32), uploads
 * GEMM weights as BF16 (norms, biases, embedding FP32) to device `ordinal`. */
J1_API j1_status j1_model_create(const char* ckpt_dir, int ordinal, j1_model** out);
J1_API void j1_model_destroy(j1_model* model);
/* "cuda:N (<device name>)"; returns the full length. */
J1_API size_t j1_model_name(const j1_model* model, char* buf, size_t cap);
J1_API j1_status j1_model_config(const j1_model* model, j1_config* out);

/* CudaModel::forward over one packed batch (model::Batch, src/model.rs:113-157):
 *   ids[t]            token ids of all sequences, back to back
 *   starts/lens[nseq] packed start row and length of each sequence (starts[s] == sum(lens[<s]))
 *   qtypes[nseq]      question type (0..2) per sequence
 *   marker_rows[m]    packed row of each option marker, grouped by sequence
 *   marker_starts[nseq+1] first marker index of each sequence, marker_starts[nseq] == m
 * scores_out[m] receives one logit per marker (flat; split with marker_starts).
 * Blocking; thread-safe (one forward at a time per model). */
J1_API j1_status j1_model_forward(j1_model* model, const uint32_t* ids, size_t t, const uint32_t* starts,
                           const uint32_t* lens, const uint8_t* qtypes, size_t nseq, const uint32_t* marker_rows,
                           const uint32_t* marker_starts, size_t m, float* scores_out);

/* The same forward split in three so a caller can keep a batch resident on the device:
 * stage (validate + pack + async H2D of the batch metadata), launch (enqueue all
 * kernels on the model's stream; may be repeated on a staged batch), finish
 * (D2H of the scores, synchronize, device-error and nonfinite checks).
 * The second launch of a batch shape (token, marker, sequence and tile counts) captures
 * its kernels into a CUDA graph that later launches of that shape replay (the same
 * kernels and results; up to 8 shapes are kept, a workspace reallocation drops them;
 * J1_GRAPH=0 in the environment turns this off). This applies to j1_model_forward and
 * the engine's forwards too. */
J1_API j1_status j1_model_stage(j1_model* model, const uint32_t* ids, size_t t, const uint32_t* starts,
                         const uint32_t* lens, const uint8_t* qtypes, size_t nseq, const uint32_t* marker_rows,
                         const uint32_t* marker_starts, size_t m);
J1_API j1_status j1_model_launch(j1_model* model);
J1_API j1_status j1_model_finish(j1_model* model, float* scores_out, size_t m);
/* cudaStream_t the model's kernels run on (for event timing by the caller). */
J1_API void* j1_model_stream(j1_model* model);

/* One packed batch, as the arguments of j1_model_forward. */
typedef struct j1_batch {
  const uint32_t* ids;
  size_t t;
  const uint32_t* starts;
  const uint32_t* lens;
  const uint8_t* qtypes;
  size_t nseq;
  const uint32_t* marker_rows;
  const uint32_t* marker_starts;
  size_t m;
} j1_batch;

/* nbatch forwards back to back, as j1_model_forward on each (scores_out[k] receives batch
 * k's m scores), pipelined: batch k+1 is validated, packed and uploaded while batch k
 * computes, and scores are read back one batch behind, so the device does not idle
 * between micro-batches (the engine's per-device loop, src/engine.rs:212-233). Every
 * batch is validated before the first launch; blocking. */
J1_API j1_status j1_model_forward_many(j1_model* model, size_t nbatch, const j1_batch* batches,
                                       float* const* scores_out);
/* Number of kernel launches one j1_model_launch issues for the staged batch. */
J1_API int64_t j1_model_launch_count(const j1_model* model);

/* Optional device timing by kernel family: with profiling on, every launch is bracketed
 * by CUDA events on the model's stream; j1_model_finish folds the elapsed times into
 * per-family totals. enable != 0 turns it on and clears the totals. */
#define J1_PROF_FAMILIES 12
J1_API j1_status j1_model_profile(j1_model* model, int enable);
/* Totals since the last j1_model_profile(model, 1): ms[J1_PROF_FAMILIES], launches[J1_PROF_FAMILIES]. */
J1_API j1_status j1_model_profile_read(j1_model* model, double* ms, int64_t* launches);
/* "embed_ln", "gemm_qkv_rope", "attn_local", "attn_global", "gemm_wo_resid_ln", "gemm_wi_geglu",
 * "gemm_wo2_resid_ln", "final_norm", "head_gemm", "head_attn", "head_gather", "scorer_gemm". */
J1_API const char* j1_profile_family_name(int family);

/* ------------------------------------------------------------ engine */
/* EngineOptions (src/engine.rs:34-65), device-side subset. */
typedef struct j1_engine_options {
  const char* device;        /* "cuda", "cuda:N" (Device::from_str, src/engine.rs:20-31); "cpu" is rejected */
  int32_t batch_size;        /* rows per forward, default 16 */
  int64_t max_batch_tokens;  /* packed tokens per forward, default 65536 */
  int32_t max_length;        /* 0 = checkpoint max_position_embeddings */
} j1_engine_options;

J1_API void j1_engine_options_default(j1_engine_options* out);
/* Engine::load on one device. */
J1_API j1_status j1_engine_create(const char* ckpt_dir, const j1_engine_options* opts, j1_engine** out);
/* Engine over n device replicas (weights replicated); micro-batches are sharded
 * across them, one host worker thread per device, logits gathered in row order. */
J1_API j1_status j1_engine_create_pool(const char* ckpt_dir, const j1_engine_options* opts, const int* ordinals, int n,
                                j1_engine** out);
J1_API void j1_engine_destroy(j1_engine* engine);
J1_API size_t j1_engine_device_name(const j1_engine* engine, char* buf, size_t cap);

/* Engine::logits_encoded (src/engine.rs:225-235) over already-encoded rows
 * (encode::Encoded: ids, marker positions within the row, qtype):
 *   ids          concatenated token ids of all rows
 *   row_lens[n]  tokens per row
 *   markers      concatenated marker positions (relative to each row's first token)
 *   row_markers[n] markers per row
 *   qtypes[n]
 * logits_out receives sum(row_markers) floats, row after row, in input order.
 * Rows are length-sorted and cut into micro-batches of at most batch_size rows
 * and max_batch_tokens tokens (src/engine.rs:191-210). */
J1_API j1_status j1_engine_logits_encoded(j1_engine* engine, size_t n_rows, const uint32_t* ids, const uint32_t* row_lens,
                                   const uint32_t* markers, const uint32_t* row_markers, const uint8_t* qtypes,
                                   float* logits_out);

/* Host-only: the micro-batch plan j1_engine_logits_encoded uses (src/engine.rs:191-210):
 * rows stable-sorted by length, cut at batch_size rows or max_batch_tokens tokens, each
 * micro-batch assigned to the replica with the fewest tokens so far.
 * batch_of_row[n_rows]; device_of_batch must hold n_rows entries (the most batches possible). */
J1_API j1_status j1_plan_batches(size_t n_rows, const uint32_t* row_lens, int32_t batch_size, int64_t max_batch_tokens,
                                 int32_t n_devices, uint32_t* batch_of_row, uint32_t* device_of_batch,
                                 size_t* n_batches);

/* The engine's row limit (EngineOptions::max_length, or the checkpoint's max_position_embeddings). */
J1_API int32_t j1_engine_max_length(const j1_engine* engine);

/* ------------------------------------------------------------ requests below the tokenizer
 * The reference turns a Request (state, question, options, qtype; src/request.rs:77-82) into
 * model rows with Encoder::sequence (src/encode.rs:138-195). Text -> token ids is the
 * caller's part (the checkpoint's tokenizer.json), using the reference's text forms:
 *   head_ids    tokens of "<choice|score|noul> question: <question>"     (encode.rs:146)
 *   option k    tokens of " <option k>"                                   (encode.rs:147)
 *   state_ids   tokens of the rendered state (State::render)              (encode.rs:180)
 * each with the mask token's text replaced by a space first (encode.rs:145); a mask id in
 * the tokens is refused ("Reserved model marker in request" in strict mode). */
typedef struct j1_encoder_options {
  uint32_t cls_id, sep_id, mask_id; /* tokenizer_config.json cls/sep/mask tokens (encode.rs:74-85) */
  int32_t max_length;               /* tokens per row; 0 = the engine's max_length (engine calls only) */
  int32_t head_length;              /* question + options budget, default 256 (engine.rs:55) */
  int32_t strict;                   /* strict_encoding: refuse instead of truncating */
} j1_encoder_options;

typedef struct j1_tokenized_request {
  const uint32_t* head_ids;
  size_t head_len;
  const uint32_t* option_ids;  /* all options' tokens, concatenated */
  const uint32_t* option_lens; /* tokens per option [n_options] */
  size_t n_options;
  const uint32_t* state_ids;
  size_t state_len;
  uint8_t qtype; /* QType: 0 choice, 1 score, 2 noul */
} j1_tokenized_request;

J1_API void j1_encoder_options_default(j1_encoder_options* out);
/* Encoder::sequence on ids: [CLS] head [SEP] ([MASK] option)... [SEP] state [SEP]; options cut
 * to 48 tokens, the head to its budget, the state to the room left. Writes the row
 * (ids_cap >= max_length), each option's marker position (markers_out[n_options]) and
 * whether the state was cut. Strict mode returns the reference's refusals instead. */
J1_API j1_status j1_encode_sequence(const j1_encoder_options* opts, const j1_tokenized_request* req,
                                    uint32_t* ids_out, size_t ids_cap, size_t* ids_len, uint32_t* markers_out,
                                    int32_t* truncated);
/* Engine::logits (src/engine.rs:236-243) on tokenized requests: Request::validate for every
 * row (2-20 options; noul = 2), encode, logits_encoded. logits_out: sum(n_options) floats. */
J1_API j1_status j1_engine_logits_tokenized(j1_engine* engine, const j1_encoder_options* opts, size_t n_rows,
                                            const j1_tokenized_request* rows, float* logits_out);

/* ------------------------------------------------------------ router
 * Router (src/router.rs): up to `width` options, one model row; larger choice requests keep
 * `survivors` per group of `width` (one if its local softmax is confident) and rerank until
 * one group remains; all groups of all requests of a call are scored together, identical
 * jobs once, and an optional LRU cache (cache_size entries) keeps logits across calls. */
typedef struct j1_router j1_router;
typedef struct j1_router_options {
  int32_t width;       /* 2..20, default 20 */
  int32_t survivors;   /* 1..width-1, default 2 */
  int32_t batch_size;  /* model rows per engine call, default 16 (the logits do not depend on it; raise it,
                          e.g. to 4096, to let the engine cut full micro-batches) */
  int32_t cache_size;  /* 0 = no cache */
  int32_t max_options; /* default 4096 */
} j1_router_options;

/* RouteResult (src/router.rs:15-26); candidates/probabilities hold n_candidates (<= width)
 * entries. probability_scope is "final_candidates" when hierarchical, else "all_options". */
typedef struct j1_route_result {
  uint32_t index;            /* chosen option, index into the request's options */
  uint32_t n_candidates;     /* options of the final group */
  uint32_t candidates[20];   /* in the order the final group was scored */
  double probabilities[20];  /* display_probabilities of the final group's softmax */
  uint32_t rounds;
  int32_t hierarchical;      /* more than width options */
} j1_route_result;

/* Scores encoded rows (layout of j1_engine_logits_encoded); returns 0 on success. */
typedef int (*j1_scorer_fn)(void* user, size_t n_rows, const uint32_t* ids, const uint32_t* row_lens,
                            const uint32_t* markers, const uint32_t* row_markers, const uint8_t* qtypes,
                            float* logits_out);

J1_API void j1_router_options_default(j1_router_options* out);
/* display_probabilities (src/request.rs:150-161): model-card rounding of probabilities. */
J1_API void j1_display_probabilities(const double* values, size_t n, double* out);
/* Router::confident_winner (src/router.rs:127-136): 1 when the group's local softmax keeps
 * only `best`. */
J1_API int32_t j1_router_confident_winner(const float* scores, size_t n, size_t best);
/* Router::new over an engine (the engine must outlive the router). */
J1_API j1_status j1_router_create(j1_engine* engine, const j1_encoder_options* enc, const j1_router_options* opts,
                                  j1_router** out);
/* The same router over a caller's scorer (e.g. another backend, or a test double). */
J1_API j1_status j1_router_create_with_scorer(j1_scorer_fn fn, void* user, const j1_encoder_options* enc,
                                              const j1_router_options* opts, j1_router** out);
J1_API void j1_router_destroy(j1_router* router);
J1_API void j1_router_clear_cache(j1_router* router);
/* Router::route_many: results[n] in request order; model_rows and cache_hits are the call's
 * totals (RouteResult::model_rows / cache_hits). */
J1_API j1_status j1_router_route_many(j1_router* router, size_t n, const j1_tokenized_request* rows,
                                      j1_route_result* results, uint64_t* model_rows, uint64_t* cache_hits);

/* ------------------------------------------------------------ text -> token ids
 * The checkpoint's tokenizer.json (byte-level BPE, the HF `tokenizers` 0.22.2 format the
 * reference loads with Tokenizer::from_bytes, src/encode.rs:55-101): added tokens, NFC
 * normalizer, ByteLevel pre-tokenizer with the GPT-2 split, BPE merges. j1_tokenizer_encode
 * returns the ids of Tokenizer::encode_fast(text, false) (src/encode.rs:114-129). Other
 * normalizers / pre-tokenizers / models are refused at load (J1_ERR_UNSUPPORTED). */
typedef struct j1_tokenizer j1_tokenizer;
J1_API j1_status j1_tokenizer_load(const char* tokenizer_json_path, j1_tokenizer** out);
J1_API j1_status j1_tokenizer_from_json(const char* json, size_t len, j1_tokenizer** out);
J1_API void j1_tokenizer_destroy(j1_tokenizer* tok);
/* Tokenizer::token_to_id; -1 when absent. */
J1_API int64_t j1_tokenizer_token_to_id(const j1_tokenizer* tok, const char* token);
/* UTF-8 text -> ids (cap entries; *n_ids is set even when cap is too small). */
J1_API j1_status j1_tokenizer_encode(const j1_tokenizer* tok, const char* text, size_t len, uint32_t* ids, size_t cap,
                                     size_t* n_ids);
/* n texts on `threads` host threads into one flat array: the ids of text i are
 * ids[offsets[i] .. offsets[i + 1]) (offsets[n + 1]). A byte-level BPE emits at most one id
 * per input byte plus one per piece for a prefix space, so cap = sum(lens) + n + 16 always
 * suffices; when cap is too small offsets[n] still holds the size needed. */
J1_API j1_status j1_tokenizer_encode_batch(const j1_tokenizer* tok, size_t n, const char* const* texts,
                                           const size_t* lens, int32_t threads, uint32_t* ids, size_t cap,
                                           size_t* offsets);

/* Encoder (src/encode.rs:25-195) on text: Encoder::load(dir, max_length, head_length, strict,
 * token_cache, encoding_cache) reads tokenizer.json and tokenizer_config.json (mask/cls/sep/pad
 * tokens); encode builds one row from the rendered state, the question, the options and the
 * qtype, with the reference's text forms, mask-token cleaning, strict refusals and LRU caches. */
typedef struct j1_text_encoder j1_text_encoder;
J1_API j1_status j1_text_encoder_load(const char* ckpt_dir, int32_t max_length, int32_t head_length, int32_t strict,
                                      int64_t token_cache, int64_t encoding_cache, j1_text_encoder** out);
J1_API void j1_text_encoder_destroy(j1_text_encoder* enc);
J1_API void j1_text_encoder_clear_cache(j1_text_encoder* enc);
/* The special ids and budgets in use (for j1_encode_sequence / j1_router_create). */
J1_API j1_status j1_text_encoder_options(const j1_text_encoder* enc, j1_encoder_options* out);
/* Encoder::tokenize: the token-fragment cache in front of the tokenizer. */
J1_API j1_status j1_text_encoder_tokenize(j1_text_encoder* enc, const char* text, size_t len, uint32_t* ids,
                                          size_t cap, size_t* n_ids);
/* Encoder::encode: state (JSON text rendered by j1_json_dumps when state_is_json, as State::render),
 * question, options[n_options] (UTF-8, NUL-terminated), qtype -> ids (cap >= max_length),
 * markers[n_options], truncated. */
J1_API j1_status j1_text_encoder_encode(j1_text_encoder* enc, const char* state, int32_t state_is_json,
                                        const char* question, const char* const* options, size_t n_options,
                                        uint8_t qtype, uint32_t* ids, size_t cap, size_t* ids_len, uint32_t* markers,
                                        int32_t* truncated);

/* State::render of a JSON state (src/pyjson.rs): Python's json.dumps(value, ensure_ascii=False)
 * byte for byte — ", " and ": " separators, key order kept, integer literals as written,
 * other numbers as float.__repr__, the json module's escapes. *out_len is set even when cap
 * is too small. */
J1_API j1_status j1_json_dumps(const char* json, size_t len, char* out, size_t cap, size_t* out_len);

/* A text request (Request, src/request.rs:77-82). With state_is_json the state is JSON text
 * (an object or an array, Request::validate), rendered with j1_json_dumps before tokenizing
 * (State::render); otherwise it is the state text itself. */
typedef struct j1_text_request {
  const char* state;
  int32_t state_is_json;
  const char* question;
  const char* const* options;
  size_t n_options;
  uint8_t qtype; /* 0 choice, 1 score, 2 noul */
} j1_text_request;
/* Engine::encode's parallel Encoder::encode (src/engine.rs:183-188) on `threads` host threads:
 * row i's ids are ids[offsets[i] .. offsets[i + 1]) and its markers markers[moffsets[i] ..];
 * cap = n * max_length and mcap = sum(n_options) always suffice; truncated[n] may be NULL.
 * The first failing row is reported as "JSONL line <i + 1>: ...". */
J1_API j1_status j1_text_encoder_encode_batch(j1_text_encoder* enc, size_t n, const j1_text_request* rows,
                                              int32_t threads, uint32_t* ids, size_t cap, size_t* offsets,
                                              uint32_t* markers, size_t mcap, size_t* moffsets, int32_t* truncated);
/* Engine::logits (src/engine.rs:236-243) on text requests: Request::validate, the parallel
 * encode above, logits_encoded. logits_out: sum(n_options) floats, row after row. */
J1_API j1_status j1_engine_logits_text(j1_engine* engine, j1_text_encoder* enc, size_t n, const j1_text_request* rows,
                                       int32_t threads, float* logits_out);

/* The tokens of a request's pieces with the text rules of Encoder::sequence (mask text
 * refused in strict mode, else replaced by a space; head "<qtype> question: <question>",
 * each " <option>", the state): ids = head | option 0 | ... | option n-1 | state, with
 * piece_lens[n_options + 2] = their lengths — a j1_tokenized_request for the router or
 * j1_engine_logits_tokenized. With ids or piece_lens NULL only *total is set. */
J1_API j1_status j1_text_encoder_request_tokens(j1_text_encoder* enc, const char* state, const char* question,
                                                const char* const* options, size_t n_options, uint8_t qtype,
                                                uint32_t* ids, size_t cap, size_t* total, uint32_t* piece_lens);

/* ------------------------------------------------------------ failure testing
 * Host-side fault injection: the next `count` device allocations (J1_FAULT_ALLOC ->
 * J1_ERR_OOM), kernel launches (J1_FAULT_LAUNCH -> J1_ERR_CUDA) or score readbacks
 * (J1_FAULT_NAN -> J1_ERR_NONFINITE, Engine::forward's check, src/engine.rs:219-221) of the
 * process fail; count 0 disarms. J1_FAULT_HOST makes the next entry points' bodies throw
 * std::bad_alloc (-> J1_ERR_OOM) and J1_FAULT_WORKER the next host worker threads (tokenizer,
 * text encoder, engine device pool) throw std::runtime_error (-> J1_ERR_INTERNAL): the paths a
 * real host failure takes. J1_FAULT_THREAD makes the next attempts to start a host worker
 * thread fail; the call then finishes its work on the threads it has (no error).
 * J1_FAULT_DEVICE_WAIT makes the next j1_op_attention_noalloc calls follow their attention
 * kernel with one bounded device wait (about 1 ms) that times out and records its site
 * (99) in the call's error word, as a timed-out wait of that kernel would. The environment
 * variable J1_FAULT=alloc|launch|nan|host|worker arms one at the first j1_model_create.
 * Nothing faults on the GPU: an injected allocation or launch does not happen, injected
 * nonfinite scores are written into the host copy, and the injected wait is bounded. */
enum { J1_FAULT_ALLOC = 1, J1_FAULT_LAUNCH = 2, J1_FAULT_NAN = 3, J1_FAULT_HOST = 4, J1_FAULT_WORKER = 5,
       J1_FAULT_THREAD = 6, J1_FAULT_DEVICE_WAIT = 7 };
J1_API void j1_inject_fault(int32_t kind, int32_t count);
/* Device-side failure detection without a fault: one thread waits, with the library's
 * bounded wait and a limit of limit_cycles (1e3..4e9), on an mbarrier nothing arrives at.
 * Returns J1_ERR_DEVICE_TIMEOUT (site 99) when the timeout was detected and reported, as a
 * forward's stuck wait would be; the context stays usable. */
J1_API j1_status j1_selftest_device_timeout(int ordinal, int64_t limit_cycles);

/* ------------------------------------------------------------ kernel-level ops
 * On caller device memory (e.g. torch tensors); `stream` is a cudaStream_t or NULL.
 * With sync != 0 the call waits for completion and reports device-side timeouts. */

/* Fused-epilogue GEMM: out = A[M,K] . W[N,K]^T, bf16 operands, fp32 accumulate. */
typedef enum j1_epilogue {
  J1_EPI_BF16 = 0,      /* out = bf16(acc (+bias)) (relu optional)                      */
  J1_EPI_QKV_ROPE = 1,  /* out = bf16(rotate_half RoPE(acc)) on columns < rope_cols     */
  J1_EPI_GEGLU = 2,     /* W rows interleaved per 128 (see j1_op_geglu_interleave);
                           out[M, N/2] = bf16(gelu(a) * b)                             */
  J1_EPI_RESID_LN = 3,  /* x[M,N] += acc (+bias) in fp32; xn = bf16(LayerNorm(x))       */
  J1_EPI_RESID = 4,     /* x[M,N] += acc (+bias)                                       */
  J1_EPI_SCORER = 5     /* scores[M] = sum_j gelu(acc + bias[j]) * w2[j] + b2           */
} j1_epilogue;

typedef struct j1_gemm_args {
  int32_t epilogue;       /* j1_epilogue */
  int32_t M, N, K;
  const void* A;          /* bf16 [M, K], row stride K */
  const void* W;          /* bf16 [N, K], row stride K */
  void* out;              /* bf16 output (BF16 / QKV_ROPE / GEGLU) */
  int32_t ldo;
  const float* bias;      /* [N] or NULL */
  int32_t relu;
  float* x;               /* fp32 residual [M, N] (RESID*) */
  int32_t ldx;
  const float* ln_w;      /* [N] */
  const float* ln_b;      /* [N] or NULL */
  float ln_eps;
  void* xn;               /* bf16 LayerNorm output */
  int32_t ldxn;
  const int32_t* pos;     /* [M] sequence position per row (QKV_ROPE) */
  const float* rope_cos;  /* [positions, 32] */
  const float* rope_sin;
  int32_t rope_cols;      /* RoPE is applied on columns < rope_cols */
  const float* w2;        /* [N] (SCORER) */
  float b2;
  float* scores;          /* [M] (SCORER) */
  int32_t grid_limit;     /* max CTAs; 0 = number of SMs */
} j1_gemm_args;

J1_API j1_status j1_op_gemm(const j1_gemm_args* args, void* stream, int sync);

/* Varlen attention over a packed qkv buffer [t, 3*hidden] (q | k | v, heads x 64 each):
 * ctx[t, hidden]. seq_starts/seq_lens are host arrays; window < 0 = full attention,
 * else |i - j| <= window (the reference's half_window). q/k are used as given
 * (RoPE is applied by J1_EPI_QKV_ROPE). */
J1_API j1_status j1_op_attention(const void* qkv, int64_t t, int32_t hidden, const uint32_t* seq_starts,
                          const uint32_t* seq_lens, size_t nseq, int32_t window, void* ctx, void* stream, int sync);

/* j1_op_attention with no run-time allocation (no counterpart in the reference).
 * Same arguments and results as j1_op_attention, but the tile list and the error words
 * live in a fixed device array of this library, so callers that cannot allocate device
 * memory (a pool that owns all free HBM; a loop that must not hit cudaMalloc's
 * device-wide synchronisation) can use it. At most 8192 query tiles (sum of
 * ceil(len / 128)) per call, else J1_ERR_INVALID_ARG. All calls on a device share that
 * array: calls on one stream are ordered, calls that overlap on the GPU (streams with no
 * ordering between them) race. CUDA places the array in device memory at the first call
 * on each device, which also does the set-up: make it (nseq = 0 does only that) before a
 * pool reserves the free memory and before any stream capture. Device-side timeouts: a
 * call with sync = 0 returns before its kernel runs, so a timeout of its kernel is
 * reported by the next call on that device made with sync = 1 (nseq = 0 with sync = 1
 * only collects), as J1_ERR_DEVICE_TIMEOUT "... in an earlier call made with sync = 0". */
J1_API j1_status j1_op_attention_noalloc(const void* qkv, int64_t t, int32_t hidden, const uint32_t* seq_starts,
                                         const uint32_t* seq_lens, size_t nseq, int32_t window, void* ctx,
                                         void* stream, int sync);

/* Host helper: dst rows of a [2*inter, K] Wi laid out for J1_EPI_GEGLU (FP32 -> BF16 on device). */
J1_API j1_status j1_op_geglu_interleave(const float* src_dev, void* dst_dev, int32_t inter, int32_t k, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* J1_H */
