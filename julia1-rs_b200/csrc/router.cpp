// The callers either side of the encoder forward, below the tokenizer:
//   * Encoder::sequence (src/encode.rs:138-195) on token ids: [CLS] head [SEP]
//     ([MASK] option)* [SEP] state [SEP], with the reference's budgets, truncation and
//     strict-mode refusals;
//   * Engine::logits (src/engine.rs:236-243) on tokenized requests: validate, encode,
//     logits_encoded;
//   * Router (src/router.rs): hierarchical choice routing over more than `width` options,
//     batching the groups of all requests of a call, with de-duplication and an optional
//     LRU cache of logits.
// Text -> ids (the checkpoint's tokenizer.json) stays with the caller.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <list>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "model.h"

using namespace j1rt;

namespace {

constexpr size_t kOptionTokens = 48;  // OPTION_TOKENS (src/encode.rs:12)

j1_status check_encoder(const j1_encoder_options* o) {
  if (!o) return set_error(J1_ERR_INVALID_ARG, "NULL encoder options");
  if (o->max_length < 1 || o->head_length < 0) return set_error(J1_ERR_INVALID_ARG, "max_length must be positive");
  // Encoder::from_parts (src/encode.rs:66-68)
  if (static_cast<int64_t>(o->head_length) + 4 >= o->max_length)
    return set_error(J1_ERR_INVALID_ARG, "max_length must leave room beyond the question head");
  return J1_OK;
}

bool has_id(const uint32_t* p, size_t n, uint32_t id) {
  for (size_t i = 0; i < n; ++i)
    if (p[i] == id) return true;
  return false;
}

// Encoder::sequence (src/encode.rs:138-195) on the request's token ids.
j1_status encode_row(const j1_encoder_options& o, const j1_tokenized_request& r, std::vector<uint32_t>& ids,
                     std::vector<uint32_t>& markers, bool& truncated) {
  if (r.n_options && !r.option_lens) return set_error(J1_ERR_INVALID_ARG, "NULL option_lens");
  size_t n_opt_tokens = 0;
  for (size_t k = 0; k < r.n_options; ++k) n_opt_tokens += r.option_lens[k];
  if ((r.head_len && !r.head_ids) || (n_opt_tokens && !r.option_ids) || (r.state_len && !r.state_ids))
    return set_error(J1_ERR_INVALID_ARG, "NULL token array");
  if (r.n_options == 0) return set_error(J1_ERR_INVALID_ARG, "request has no options");
  // The reference replaces the mask token's text before tokenizing, or refuses it in
  // strict mode (encode.rs:141-144); on ids the mask id can only come from that text.
  if (has_id(r.head_ids, r.head_len, o.mask_id) || has_id(r.option_ids, n_opt_tokens, o.mask_id) ||
      has_id(r.state_ids, r.state_len, o.mask_id))
    return set_error(J1_ERR_INVALID_ARG, o.strict ? "Reserved model marker in request"
                                                  : "mask token id inside request tokens (replace the mask "
                                                    "token's text before tokenizing)");
  std::vector<std::vector<uint32_t>> options(r.n_options);
  size_t off = 0;
  for (size_t k = 0; k < r.n_options; ++k) {
    const size_t n = r.option_lens[k];
    if (o.strict && n > kOptionTokens) return set_error(J1_ERR_INVALID_ARG, "Option exceeds 48-token model contract");
    options[k].push_back(o.mask_id);
    options[k].insert(options[k].end(), r.option_ids + off, r.option_ids + off + std::min(n, kOptionTokens));
    off += n;
  }
  auto used = [&]() {
    int64_t s = 0;
    for (const auto& v : options) s += static_cast<int64_t>(v.size());
    return s;
  };
  const int64_t head_length = o.head_length;
  int64_t budget = head_length - used();
  if (budget < 16) {
    // (head_length - 16).div_euclid(n).max(4)
    const int64_t n = static_cast<int64_t>(options.size());
    const int64_t a = head_length - 16;
    int64_t q = a / n;
    if (a % n != 0 && a < 0) --q;
    const size_t per_option = static_cast<size_t>(std::max<int64_t>(q, 4));
    for (auto& v : options)
      if (v.size() > per_option) v.resize(per_option);
    budget = head_length - used();
  }
  if (o.strict) {
    bool cut = static_cast<int64_t>(r.head_len) > budget;
    for (size_t k = 0; k < r.n_options && !cut; ++k) cut = options[k].size() != r.option_lens[k] + 1;
    if (cut) return set_error(J1_ERR_INVALID_ARG, "Question/options exceed lossless head budget");
  }
  ids.clear();
  markers.clear();
  ids.push_back(o.cls_id);
  const size_t head_keep = std::min<size_t>(r.head_len, static_cast<size_t>(std::max<int64_t>(budget, 8)));
  ids.insert(ids.end(), r.head_ids, r.head_ids + head_keep);
  ids.push_back(o.sep_id);
  for (const auto& v : options) {
    markers.push_back(static_cast<uint32_t>(ids.size()));
    ids.insert(ids.end(), v.begin(), v.end());
  }
  ids.push_back(o.sep_id);
  const int64_t room = static_cast<int64_t>(o.max_length) - static_cast<int64_t>(ids.size()) - 1;
  if (room < 1) return set_error(J1_ERR_INVALID_ARG, "Question/options exceed sequence budget; shorten descriptions");
  if (o.strict && static_cast<int64_t>(r.state_len) > room)
    return set_error(J1_ERR_INVALID_ARG, "Game state exceeds lossless context budget");
  const size_t state_keep = std::min<size_t>(r.state_len, static_cast<size_t>(room));
  ids.insert(ids.end(), r.state_ids, r.state_ids + state_keep);
  ids.push_back(o.sep_id);
  truncated = static_cast<int64_t>(r.state_len) > room;
  return J1_OK;
}

// Request::validate (src/request.rs:132-146), on what survives tokenization.
j1_status validate_request(const j1_tokenized_request& r) {
  bool empty = false;
  for (size_t k = 0; k < r.n_options && r.option_lens; ++k) empty = empty || r.option_lens[k] == 0;
  if (r.n_options < 2 || r.n_options > 20 || empty)
    return set_error(J1_ERR_INVALID_ARG, "options must contain 2–20 nonempty rendered descriptions");
  if (r.qtype > 2) return set_error(J1_ERR_INVALID_ARG, "qtype must be 0 (choice), 1 (score) or 2 (noul)");
  if (r.qtype == 2 && r.n_options != 2) return set_error(J1_ERR_INVALID_ARG, "noul options must be ordered [false, true]");
  return J1_OK;
}

// Encoded rows in the layout of j1_engine_logits_encoded.
struct EncodedRows {
  std::vector<uint32_t> ids, lens, markers, nmark;
  std::vector<uint8_t> qtypes;
  size_t n = 0;
  j1_status add(const j1_encoder_options& o, const j1_tokenized_request& r) {
    std::vector<uint32_t> row, mk;
    bool trunc = false;
    if (j1_status s = encode_row(o, r, row, mk, trunc)) return s;
    ids.insert(ids.end(), row.begin(), row.end());
    lens.push_back(static_cast<uint32_t>(row.size()));
    markers.insert(markers.end(), mk.begin(), mk.end());
    nmark.push_back(static_cast<uint32_t>(mk.size()));
    qtypes.push_back(r.qtype);
    ++n;
    return J1_OK;
  }
};

// A request restricted to a subset of its options (the router's group jobs).
struct Job {
  const j1_tokenized_request* row;
  std::vector<uint32_t> opt_ids, opt_lens;
  j1_tokenized_request view() const {
    j1_tokenized_request v = *row;
    v.option_ids = opt_ids.data();
    v.option_lens = opt_lens.data();
    v.n_options = opt_lens.size();
    return v;
  }
};

// argmax (src/request.rs:164-172): first index of the maximum.
template <typename T>
size_t argmax(const T* v, size_t n) {
  size_t best = 0;
  for (size_t i = 0; i < n; ++i)
    if (v[i] > v[best]) best = i;
  return best;
}

// display_probabilities (src/request.rs:150-161).
std::vector<double> display_probabilities(const std::vector<double>& values) {
  if (values.empty()) return {};
  const size_t w = argmax(values.data(), values.size());
  bool one_hot = values[w] > 0.95;
  for (size_t i = 0; i < values.size() && one_hot; ++i) one_hot = i == w || values[i] < 0.045;
  std::vector<double> out(values.size(), 0.0);
  if (one_hot) {
    out[w] = 1.0;
    return out;
  }
  double total = 0.0;
  for (size_t i = 0; i < values.size(); ++i) {
    out[i] = values[i] >= 0.01 ? values[i] : 0.0;
    total += out[i];
  }
  for (double& v : out) v /= total;
  return out;
}

// Router::confident_winner (src/router.rs:127-136).
bool confident_winner(const std::vector<float>& scores, size_t best) {
  const double sb = scores[best];
  double runner_up = -INFINITY;
  for (size_t i = 0; i < scores.size(); ++i)
    if (i != best) runner_up = std::max(runner_up, static_cast<double>(scores[i]));
  if (runner_up - sb >= std::log(0.045 / 0.95)) return false;
  double total = 0.0;
  for (float v : scores) total += std::exp(static_cast<double>(v) - sb);
  return 1.0 / total > 0.95 && std::exp(runner_up - sb) / total < 0.045;
}

}  // namespace

struct j1_router {
  j1_engine* engine = nullptr;
  j1_scorer_fn scorer = nullptr;
  void* user = nullptr;
  j1_encoder_options enc{};
  j1_router_options opts{};
  // LRU cache of logits by request key (lru::LruCache semantics: get promotes, put
  // evicts the least recently used entry once full)
  std::list<std::pair<std::string, std::vector<float>>> lru;
  std::unordered_map<std::string, std::list<std::pair<std::string, std::vector<float>>>::iterator> lru_index;
  std::mutex lock;  // Router::lock: one route_many at a time

  const std::vector<float>* cache_get(const std::string& key) {
    auto it = lru_index.find(key);
    if (it == lru_index.end()) return nullptr;
    lru.splice(lru.begin(), lru, it->second);
    return &it->second->second;
  }
  void cache_put(const std::string& key, const std::vector<float>& v) {
    if (opts.cache_size <= 0) return;
    auto it = lru_index.find(key);
    if (it != lru_index.end()) {
      it->second->second = v;
      lru.splice(lru.begin(), lru, it->second);
      return;
    }
    if (lru.size() >= static_cast<size_t>(opts.cache_size)) {
      lru_index.erase(lru.back().first);
      lru.pop_back();
    }
    lru.emplace_front(key, v);
    lru_index[key] = lru.begin();
  }

  // Logits of encoded rows from the engine or the caller's scorer.
  j1_status logits(const EncodedRows& rows, std::vector<float>& out) {
    size_t m = 0;
    for (uint32_t k : rows.nmark) m += k;
    out.assign(m, 0.f);
    if (rows.n == 0) return J1_OK;
    if (engine)
      return j1_engine_logits_encoded(engine, rows.n, rows.ids.data(), rows.lens.data(), rows.markers.data(),
                                      rows.nmark.data(), rows.qtypes.data(), out.data());
    const int rc = scorer(user, rows.n, rows.ids.data(), rows.lens.data(), rows.markers.data(), rows.nmark.data(),
                          rows.qtypes.data(), out.data());
    if (rc != 0) return set_error(J1_ERR_INVALID_ARG, "scorer callback failed (" + std::to_string(rc) + ")");
    return J1_OK;
  }
};

namespace {

// Router::key (src/router.rs:87-89): everything the logits depend on.
std::string job_key(const Job& j) {
  std::string k;
  auto put = [&k](const void* p, size_t bytes) { k.append(static_cast<const char*>(p), bytes); };
  const uint64_t hl = j.row->head_len, sl = j.row->state_len, no = j.opt_lens.size();
  put(&j.row->qtype, 1);
  put(&hl, 8);
  put(j.row->head_ids, hl * 4);
  put(&sl, 8);
  put(j.row->state_ids, sl * 4);
  put(&no, 8);
  put(j.opt_lens.data(), no * 4);
  put(j.opt_ids.data(), j.opt_ids.size() * 4);
  return k;
}

// Router::score (src/router.rs:91-124): cache hits, de-duplication inside the call, then
// one model row per distinct job, batch_size rows per engine call. The logits do not
// depend on batch_size (a row's forward does not depend on the other rows of its batch);
// a large batch_size lets the engine cut full micro-batches for the devices.
j1_status score(j1_router* R, const std::vector<Job>& jobs, std::vector<std::vector<float>>& values,
                size_t& used, size_t& hits) {
  values.assign(jobs.size(), {});
  std::vector<std::pair<std::string, std::vector<size_t>>> missing;
  std::unordered_map<std::string, size_t> index;
  std::vector<char> have(jobs.size(), 0);
  hits = 0;
  for (size_t i = 0; i < jobs.size(); ++i) {
    std::string key = job_key(jobs[i]);
    if (R->opts.cache_size > 0) {
      if (const std::vector<float>* v = R->cache_get(key)) {
        values[i] = *v;
        have[i] = 1;
        ++hits;
        continue;
      }
    }
    auto it = index.find(key);
    if (it != index.end()) {
      missing[it->second].second.push_back(i);
      ++hits;
    } else {
      index.emplace(key, missing.size());
      missing.emplace_back(std::move(key), std::vector<size_t>{i});
    }
  }
  const size_t chunk = static_cast<size_t>(R->opts.batch_size);
  for (size_t c0 = 0; c0 < missing.size(); c0 += chunk) {
    const size_t c1 = std::min(missing.size(), c0 + chunk);
    EncodedRows rows;
    for (size_t q = c0; q < c1; ++q) {
      const j1_tokenized_request v = jobs[missing[q].second[0]].view();
      if (j1_status s = validate_request(v)) return s;
      if (j1_status s = rows.add(R->enc, v)) return s;
    }
    std::vector<float> flat;
    if (j1_status s = R->logits(rows, flat)) return s;
    size_t o = 0;
    for (size_t q = c0; q < c1; ++q) {
      const size_t n = rows.nmark[q - c0];
      std::vector<float> sc(flat.begin() + o, flat.begin() + o + n);
      o += n;
      for (float v : sc)
        if (!std::isfinite(v))
          return set_error(J1_ERR_NONFINITE, "Engine logits must be finite and match option count");
      for (size_t i : missing[q].second) values[i] = sc;
      R->cache_put(missing[q].first, sc);
    }
  }
  used = missing.size();
  return J1_OK;
}

j1_status validate_route(const j1_router* R, const j1_tokenized_request& r) {
  if (r.n_options < 2 || r.n_options > static_cast<size_t>(R->opts.max_options))
    return set_error(J1_ERR_INVALID_ARG, "Expected 2–" + std::to_string(R->opts.max_options) + " options");
  if (!r.option_lens) return set_error(J1_ERR_INVALID_ARG, "NULL option_lens");
  for (size_t k = 0; k < r.n_options; ++k)
    if (r.option_lens[k] == 0) return set_error(J1_ERR_INVALID_ARG, "Options must be nonempty strings");
  if (r.qtype > 2) return set_error(J1_ERR_INVALID_ARG, "qtype must be 0 (choice), 1 (score) or 2 (noul)");
  if (r.qtype == 2 && r.n_options != 2) return set_error(J1_ERR_INVALID_ARG, "noul requires [false, true]");
  if (r.qtype != 0 && r.n_options > static_cast<size_t>(R->opts.width))
    return set_error(J1_ERR_INVALID_ARG, "Hierarchical routing supports choice decisions only");
  return J1_OK;
}

j1_status make_router(j1_engine* engine, j1_scorer_fn fn, void* user, const j1_encoder_options* enc,
                      const j1_router_options* opts, j1_router** out) {
  if (!out || !enc) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
  *out = nullptr;
  j1_router_options o;
  j1_router_options_default(&o);
  if (opts) o = *opts;
  // Router::new (src/router.rs:39-55)
  if (o.width < 2 || o.width > 20 || o.survivors < 1 || o.survivors >= o.width)
    return set_error(J1_ERR_INVALID_ARG, "Require 2 <= width <= 20 and 1 <= survivors < width");
  if (o.batch_size < 1 || o.max_options < o.width || o.cache_size < 0)
    return set_error(J1_ERR_INVALID_ARG, "Invalid batch/cache/capacity limit");
  j1_encoder_options e = *enc;
  if (engine && e.max_length == 0) e.max_length = j1_engine_max_length(engine);
  if (j1_status s = check_encoder(&e)) return s;
  if (engine && e.max_length > j1_engine_max_length(engine))
    return set_error(J1_ERR_INVALID_ARG, "encoder max_length exceeds the engine's max_length");
  auto R = std::make_unique<j1_router>();
  R->engine = engine;
  R->scorer = fn;
  R->user = user;
  R->enc = e;
  R->opts = o;
  *out = R.release();
  return J1_OK;
}

}  // namespace

extern "C" {

void j1_encoder_options_default(j1_encoder_options* o) {
  if (!o) return;
  *o = j1_encoder_options{};
  o->max_length = 0;    // engine calls: the engine's max_length (checkpoint max_position_embeddings)
  o->head_length = 256;  // EngineOptions::default (src/engine.rs:55)
  o->strict = 0;
}

j1_status j1_encode_sequence(const j1_encoder_options* opts, const j1_tokenized_request* req, uint32_t* ids_out,
                             size_t ids_cap, size_t* ids_len, uint32_t* markers_out, int32_t* truncated) {
  return guard("j1_encode_sequence", [&]() -> j1_status {
    if (!req || !ids_len) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (j1_status s = check_encoder(opts)) return s;
    std::vector<uint32_t> ids, mk;
    bool trunc = false;
    if (j1_status s = encode_row(*opts, *req, ids, mk, trunc)) return s;
    if (ids.size() > ids_cap || !ids_out || (!markers_out && !mk.empty()))
      return set_error(J1_ERR_INVALID_ARG, "output arrays too small (ids_cap >= max_length, markers >= n_options)");
    std::memcpy(ids_out, ids.data(), ids.size() * 4);
    if (!mk.empty()) std::memcpy(markers_out, mk.data(), mk.size() * 4);
    *ids_len = ids.size();
    if (truncated) *truncated = trunc ? 1 : 0;
    return J1_OK;
  });
}

j1_status j1_engine_logits_tokenized(j1_engine* engine, const j1_encoder_options* opts, size_t n_rows,
                                     const j1_tokenized_request* rows, float* logits_out) {
  return guard("j1_engine_logits_tokenized", [&]() -> j1_status {
    if (!engine || !opts) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (n_rows == 0) return J1_OK;
    if (!rows || !logits_out) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    j1_encoder_options e = *opts;
    if (e.max_length == 0) e.max_length = j1_engine_max_length(engine);
    if (j1_status s = check_encoder(&e)) return s;
    // Engine::encode (src/engine.rs:183-188): validate every row before encoding any
    for (size_t i = 0; i < n_rows; ++i)
      if (j1_status s = validate_request(rows[i]))
        return set_error(s, "JSONL line " + std::to_string(i + 1) + ": " + [] {
          char buf[256];
          j1_last_error(buf, sizeof(buf));
          return std::string(buf);
        }());
    EncodedRows enc;
    for (size_t i = 0; i < n_rows; ++i)
      if (j1_status s = enc.add(e, rows[i])) return s;
    return j1_engine_logits_encoded(engine, enc.n, enc.ids.data(), enc.lens.data(), enc.markers.data(),
                                    enc.nmark.data(), enc.qtypes.data(), logits_out);
  });
}

void j1_display_probabilities(const double* values, size_t n, double* out) {
  if (!values || !out) return;
  const j1_status s = guard("j1_display_probabilities", [&]() -> j1_status {
    const std::vector<double> p = display_probabilities(std::vector<double>(values, values + n));
    std::copy(p.begin(), p.end(), out);
    return J1_OK;
  });
  if (s)  // host memory exhausted: no probabilities (the message is in j1_last_error)
    for (size_t i = 0; i < n; ++i) out[i] = std::numeric_limits<double>::quiet_NaN();
}

int32_t j1_router_confident_winner(const float* scores, size_t n, size_t best) {
  if (!scores || best >= n) return 0;
  int32_t win = 0;
  guard("j1_router_confident_winner", [&]() -> j1_status {
    win = confident_winner(std::vector<float>(scores, scores + n), best) ? 1 : 0;
    return J1_OK;
  });
  return win;
}

void j1_router_options_default(j1_router_options* o) {
  if (!o) return;
  // Router::with_defaults (src/router.rs:57-60)
  o->width = 20;
  o->survivors = 2;
  o->batch_size = 16;
  o->cache_size = 0;
  o->max_options = 4096;
}

j1_status j1_router_create(j1_engine* engine, const j1_encoder_options* enc, const j1_router_options* opts,
                           j1_router** out) {
  return guard("j1_router_create", [&]() -> j1_status {
    if (!engine) return set_error(J1_ERR_INVALID_ARG, "NULL engine");
    return make_router(engine, nullptr, nullptr, enc, opts, out);
  });
}

j1_status j1_router_create_with_scorer(j1_scorer_fn fn, void* user, const j1_encoder_options* enc,
                                       const j1_router_options* opts, j1_router** out) {
  return guard("j1_router_create_with_scorer", [&]() -> j1_status {
    if (!fn) return set_error(J1_ERR_INVALID_ARG, "NULL scorer");
    return make_router(nullptr, fn, user, enc, opts, out);
  });
}

void j1_router_destroy(j1_router* r) { delete r; }

void j1_router_clear_cache(j1_router* r) {
  if (!r) return;
  std::lock_guard<std::mutex> lk(r->lock);
  r->lru.clear();
  r->lru_index.clear();
}

// Router::route_many (src/router.rs:143-210).
j1_status j1_router_route_many(j1_router* R, size_t n, const j1_tokenized_request* rows, j1_route_result* results,
                               uint64_t* model_rows, uint64_t* cache_hits) {
  return guard("j1_router_route_many", [&]() -> j1_status {
    if (!R) return set_error(J1_ERR_INVALID_ARG, "NULL router");
    if (n && (!rows || !results)) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::lock_guard<std::mutex> lk(R->lock);
    for (size_t i = 0; i < n; ++i)
      if (j1_status s = validate_route(R, rows[i])) return s;
    const size_t width = static_cast<size_t>(R->opts.width);
    // per row: offsets of each option's tokens
    std::vector<std::vector<size_t>> opt_off(n);
    for (size_t i = 0; i < n; ++i) {
      opt_off[i].assign(rows[i].n_options + 1, 0);
      for (size_t k = 0; k < rows[i].n_options; ++k) opt_off[i][k + 1] = opt_off[i][k] + rows[i].option_lens[k];
    }
    std::vector<std::vector<uint32_t>> candidates(n);
    for (size_t i = 0; i < n; ++i)
      for (size_t k = 0; k < rows[i].n_options; ++k) candidates[i].push_back(static_cast<uint32_t>(k));
    std::vector<char> done(n, 0);
    std::vector<uint32_t> rounds(n, 0);
    size_t used_total = 0, hits_total = 0, remaining = n;
    struct Slot {
      size_t row;
      std::vector<uint32_t> group;
      bool last;
    };
    while (remaining > 0) {
      std::vector<Job> jobs;
      std::vector<Slot> layout;
      for (size_t i = 0; i < n; ++i) {
        if (done[i]) continue;
        ++rounds[i];
        std::vector<uint32_t> current;
        current.swap(candidates[i]);
        const bool last = current.size() <= width;
        for (size_t g0 = 0; g0 < current.size(); g0 += width) {
          const size_t g1 = std::min(current.size(), g0 + width);
          if (g1 - g0 == 1) {
            candidates[i].push_back(current[g0]);
            continue;
          }
          Job j;
          j.row = &rows[i];
          std::vector<uint32_t> group(current.begin() + g0, current.begin() + g1);
          for (uint32_t k : group) {
            j.opt_lens.push_back(rows[i].option_lens[k]);
            j.opt_ids.insert(j.opt_ids.end(), rows[i].option_ids + opt_off[i][k], rows[i].option_ids + opt_off[i][k + 1]);
          }
          jobs.push_back(std::move(j));
          layout.push_back(Slot{i, std::move(group), last});
        }
      }
      std::vector<std::vector<float>> scored;
      size_t used = 0, hits = 0;
      if (j1_status s = score(R, jobs, scored, used, hits)) return s;
      used_total += used;
      hits_total += hits;
      for (size_t q = 0; q < layout.size(); ++q) {
        const Slot& sl = layout[q];
        const std::vector<float>& sc = scored[q];
        const size_t best = argmax(sc.data(), sc.size());
        const size_t i = sl.row;
        if (sl.last) {
          double mx = -INFINITY;
          for (float v : sc) mx = std::max(mx, static_cast<double>(v));
          std::vector<double> w(sc.size());
          double total = 0.0;
          for (size_t k = 0; k < sc.size(); ++k) {
            w[k] = std::exp(static_cast<double>(sc[k]) - mx);
            total += w[k];
          }
          for (double& v : w) v /= total;
          const std::vector<double> p = display_probabilities(w);
          j1_route_result& res = results[i];
          std::memset(&res, 0, sizeof(res));
          res.index = sl.group[best];
          res.n_candidates = static_cast<uint32_t>(sl.group.size());
          for (size_t k = 0; k < sl.group.size(); ++k) {
            res.candidates[k] = sl.group[k];
            res.probabilities[k] = p[k];
          }
          res.rounds = rounds[i];
          res.hierarchical = rows[i].n_options > width ? 1 : 0;
          done[i] = 1;
          --remaining;
        } else if (confident_winner(sc, best)) {
          candidates[i].push_back(sl.group[best]);
        } else {
          std::vector<size_t> rest(sl.group.size());
          for (size_t k = 0; k < rest.size(); ++k) rest[k] = k;
          std::vector<uint32_t> chosen;
          const size_t keep = std::min(static_cast<size_t>(R->opts.survivors), sl.group.size());
          for (size_t c = 0; c < keep; ++c) {
            std::vector<float> local(rest.size());
            for (size_t k = 0; k < rest.size(); ++k) local[k] = sc[rest[k]];
            const size_t a = argmax(local.data(), local.size());
            chosen.push_back(sl.group[rest[a]]);
            rest.erase(rest.begin() + static_cast<std::ptrdiff_t>(a));
          }
          std::sort(chosen.begin(), chosen.end());
          candidates[i].insert(candidates[i].end(), chosen.begin(), chosen.end());
        }
      }
    }
    if (model_rows) *model_rows = used_total;
    if (cache_hits) *cache_hits = hits_total;
    return J1_OK;
  });
}

}  // extern "C"
