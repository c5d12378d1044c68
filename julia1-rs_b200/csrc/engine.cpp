// Engine: Engine::logits_encoded semantics (src/engine.rs:190-235) over one or
// more device replicas. Rows are length-sorted and cut into micro-batches
// (batch_size rows, max_batch_tokens tokens); with several replicas the
// micro-batches are dealt out by greedy token balance, one host worker thread
// per device, and the logits are written back in the caller's row order.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <memory>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "model.h"

using namespace j1rt;

struct j1_engine {
  std::vector<j1_model*> models;
  j1_engine_options opts;
  int max_length = 0;
  std::string name;
  std::mutex mu;  // Engine::lock (src/engine.rs:78,226)
};

namespace {

j1_status parse_device(const char* s, int* ordinal) {
  const std::string d = s ? s : "cuda";
  if (d == "cpu")
    return set_error(J1_ERR_UNSUPPORTED, "libj1 is the CUDA (sm_100a) backend; it has no CPU fallback");
  if (d == "cuda") {
    *ordinal = 0;
    return J1_OK;
  }
  if (d.rfind("cuda:", 0) == 0 && d.size() > 5) {
    const std::string n = d.substr(5);
    if (n.find_first_not_of("0123456789") == std::string::npos && n.size() < 6) {
      *ordinal = std::stoi(n);
      return J1_OK;
    }
  }
  return set_error(J1_ERR_INVALID_ARG, "device must be cpu, cuda or cuda:N");
}

j1_status check_options(j1_engine* e, const ModelConfig& c) {
  const int ml = e->opts.max_length > 0 ? e->opts.max_length : c.max_positions;
  if (ml < 1 || ml > c.max_positions)
    return set_error(J1_ERR_INVALID_ARG,
                     "max_length must be an integer between 1 and " + std::to_string(c.max_positions));
  if (e->opts.batch_size < 1 || e->opts.max_batch_tokens < ml)
    return set_error(J1_ERR_INVALID_ARG, "Invalid batch size / token budget");
  e->max_length = ml;
  return J1_OK;
}

struct Micro {
  std::vector<size_t> rows;
  size_t tokens = 0;
};

// Engine::batches (src/engine.rs:191-210): rows sorted by length (stable), cut when a
// micro-batch reaches batch_size rows or would exceed max_batch_tokens. Then each
// micro-batch goes to the replica with the fewest tokens so far (ties: lowest index).
void plan(size_t n_rows, const uint32_t* row_lens, size_t batch_size, size_t max_batch_tokens, size_t n_devices,
          std::vector<Micro>& micro, std::vector<size_t>& device_of) {
  std::vector<size_t> order(n_rows);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return row_lens[a] < row_lens[b]; });
  micro.clear();
  Micro cur;
  for (size_t i : order) {
    const size_t n = row_lens[i];
    if (!cur.rows.empty() && (cur.rows.size() == batch_size || cur.tokens + n > max_batch_tokens)) {
      micro.push_back(std::move(cur));
      cur = Micro();
    }
    cur.rows.push_back(i);
    cur.tokens += n;
  }
  if (!cur.rows.empty()) micro.push_back(std::move(cur));
  std::vector<size_t> load(n_devices, 0);
  device_of.assign(micro.size(), 0);
  for (size_t b = 0; b < micro.size(); ++b) {
    const size_t g = static_cast<size_t>(std::min_element(load.begin(), load.end()) - load.begin());
    device_of[b] = g;
    load[g] += micro[b].tokens;
  }
}

}  // namespace

size_t j1rt::engine_pipeline_rows(const j1_engine* e) {
  const size_t b = e->opts.batch_size > 0 ? static_cast<size_t>(e->opts.batch_size) : 16;
  return std::max<size_t>(256, 4 * b * std::max<size_t>(e->models.size(), 1));
}

extern "C" {

void j1_engine_options_default(j1_engine_options* o) {
  if (!o) return;
  o->device = "cuda";
  o->batch_size = 16;
  o->max_batch_tokens = 65536;
  o->max_length = 0;
}

j1_status j1_engine_create_pool(const char* ckpt_dir, const j1_engine_options* opts, const int* ordinals, int n,
                                j1_engine** out) {
  return guard("j1_engine_create_pool", [&]() -> j1_status {
    if (!ckpt_dir || !out || n < 1 || !ordinals) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    std::unique_ptr<j1_engine> e(new j1_engine());
    if (opts) e->opts = *opts;
    else j1_engine_options_default(&e->opts);
    e->opts.device = nullptr;  // not retained
    for (int i = 0; i < n; ++i) {
      j1_model* m = nullptr;
      j1_status s = j1_model_create(ckpt_dir, ordinals[i], &m);
      if (s) {
        for (auto* x : e->models) j1_model_destroy(x);
        return s;
      }
      e->models.push_back(m);
    }
    j1_status s = check_options(e.get(), e->models[0]->cfg);
    if (s) {
      for (auto* x : e->models) j1_model_destroy(x);
      return s;
    }
    for (size_t i = 0; i < e->models.size(); ++i) e->name += (i ? ", " : "") + e->models[i]->name;
    *out = e.release();
    return J1_OK;
  });
}

j1_status j1_engine_create(const char* ckpt_dir, const j1_engine_options* opts, j1_engine** out) {
  return guard("j1_engine_create", [&]() -> j1_status {
    int ordinal = 0;
    j1_status s = parse_device(opts ? opts->device : "cuda", &ordinal);
    if (s) return s;
    return j1_engine_create_pool(ckpt_dir, opts, &ordinal, 1, out);
  });
}

void j1_engine_destroy(j1_engine* e) {
  if (!e) return;
  for (auto* m : e->models) j1_model_destroy(m);
  delete e;
}

size_t j1_engine_device_name(const j1_engine* e, char* buf, size_t cap) {
  const size_t n = e ? e->name.size() : 0;  // no allocation here
  if (buf && cap) {
    const size_t k = n < cap - 1 ? n : cap - 1;
    if (k) std::memcpy(buf, e->name.data(), k);
    buf[k] = 0;
  }
  return n;
}

j1_status j1_engine_logits_encoded(j1_engine* e, size_t n_rows, const uint32_t* ids, const uint32_t* row_lens,
                                   const uint32_t* markers, const uint32_t* row_markers, const uint8_t* qtypes,
                                   float* logits_out) {
  return guard("j1_engine_logits_encoded", [&]() -> j1_status {
    if (!e) return set_error(J1_ERR_INVALID_ARG, "NULL engine");
    if (n_rows == 0) return J1_OK;
    if (!ids || !row_lens || !row_markers || !qtypes) return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    std::vector<size_t> tok_off(n_rows + 1, 0), mk_off(n_rows + 1, 0);
    for (size_t r = 0; r < n_rows; ++r) {
      if (row_lens[r] == 0 || row_lens[r] > static_cast<uint32_t>(e->max_length))
        return set_error(J1_ERR_INVALID_ARG,
                         "row " + std::to_string(r + 1) + ": length must be in 1.." + std::to_string(e->max_length));
      if (qtypes[r] > 2) return set_error(J1_ERR_INVALID_ARG, "qtype must be 0, 1 or 2");
      tok_off[r + 1] = tok_off[r] + row_lens[r];
      mk_off[r + 1] = mk_off[r] + row_markers[r];
    }
    if (mk_off[n_rows] && (!markers || !logits_out)) return set_error(J1_ERR_INVALID_ARG, "NULL markers/logits");
    for (size_t r = 0; r < n_rows; ++r)
      for (size_t k = mk_off[r]; k < mk_off[r + 1]; ++k)
        if (markers[k] >= row_lens[r]) return set_error(J1_ERR_INVALID_ARG, "marker outside its row");

    std::lock_guard<std::mutex> lk(e->mu);
    const size_t G = e->models.size();
    std::vector<Micro> micro;
    std::vector<size_t> device_of;
    plan(n_rows, row_lens, static_cast<size_t>(e->opts.batch_size), static_cast<size_t>(e->opts.max_batch_tokens), G,
         micro, device_of);
    std::vector<std::vector<size_t>> assign(G);
    for (size_t b = 0; b < micro.size(); ++b) assign[device_of[b]].push_back(b);

    // One worker per replica packs its micro-batches (Batch::new, src/model.rs:225-269) and
    // runs them through j1_model_forward_many, which overlaps the staging of batch k+1
    // with the forward of batch k; logits go back in the caller's row order.
    struct Packed {
      std::vector<uint32_t> ids, starts, lens, mrows, mstarts;
      std::vector<uint8_t> qt;
      std::vector<float> scores;
    };
    auto run = [&](size_t g, j1_status* status, std::string* msg) {
      std::vector<Packed> pk(assign[g].size());
      std::vector<j1_batch> jb(pk.size());
      std::vector<float*> outs(pk.size());
      for (size_t i = 0; i < pk.size(); ++i) {
        const Micro& mb = micro[assign[g][i]];
        Packed& P = pk[i];
        P.mstarts.assign(1, 0);
        for (size_t r : mb.rows) {
          const uint32_t start = static_cast<uint32_t>(P.ids.size());
          P.starts.push_back(start);
          P.lens.push_back(row_lens[r]);
          P.qt.push_back(qtypes[r]);
          P.ids.insert(P.ids.end(), ids + tok_off[r], ids + tok_off[r + 1]);
          for (size_t k = mk_off[r]; k < mk_off[r + 1]; ++k) P.mrows.push_back(start + markers[k]);
          P.mstarts.push_back(static_cast<uint32_t>(P.mrows.size()));
        }
        P.scores.assign(P.mrows.size(), 0.f);
        jb[i] = j1_batch{P.ids.data(), P.ids.size(), P.starts.data(), P.lens.data(), P.qt.data(), P.starts.size(),
                         P.mrows.data(), P.mstarts.data(), P.mrows.size()};
        outs[i] = P.scores.data();
      }
      j1_status s = j1_model_forward_many(e->models[g], jb.size(), jb.data(), outs.data());
      if (s) {
        *status = s;
        char buf[512];
        j1_last_error(buf, sizeof(buf));
        *msg = buf;
        return;
      }
      for (size_t i = 0; i < pk.size(); ++i) {
        size_t k = 0;
        for (size_t r : micro[assign[g][i]].rows)
          for (size_t j = mk_off[r]; j < mk_off[r + 1]; ++j) logits_out[j] = pk[i].scores[k++];
      }
    };

    std::vector<j1_status> st(G, J1_OK);
    std::vector<std::string> msgs(G);
    std::atomic<size_t> next_device{0};  // one worker per device while threads can be had
    run_pool(static_cast<int>(G), [&] {
      for (size_t g = next_device++; g < G; g = next_device++) run(g, &st[g], &msgs[g]);
    });
    for (size_t g = 0; g < G; ++g)
      if (st[g]) return set_error(st[g], msgs[g]);
    return J1_OK;
  });
}

int32_t j1_engine_max_length(const j1_engine* e) { return e ? e->max_length : 0; }

j1_status j1_plan_batches(size_t n_rows, const uint32_t* row_lens, int32_t batch_size, int64_t max_batch_tokens,
                          int32_t n_devices, uint32_t* batch_of_row, uint32_t* device_of_batch, size_t* n_batches) {
  return guard("j1_plan_batches", [&]() -> j1_status {
    if (!n_batches || (n_rows && (!row_lens || !batch_of_row || !device_of_batch)))
      return set_error(J1_ERR_INVALID_ARG, "NULL argument");
    if (batch_size < 1 || max_batch_tokens < 1 || n_devices < 1)
      return set_error(J1_ERR_INVALID_ARG, "batch_size, max_batch_tokens and n_devices must be positive");
    std::vector<Micro> micro;
    std::vector<size_t> device_of;
    plan(n_rows, row_lens, static_cast<size_t>(batch_size), static_cast<size_t>(max_batch_tokens),
         static_cast<size_t>(n_devices), micro, device_of);
    for (size_t b = 0; b < micro.size(); ++b) {
      device_of_batch[b] = static_cast<uint32_t>(device_of[b]);
      for (size_t r : micro[b].rows) batch_of_row[r] = static_cast<uint32_t>(b);
    }
    *n_batches = micro.size();
    return J1_OK;
  });
}

}  // extern "C"
