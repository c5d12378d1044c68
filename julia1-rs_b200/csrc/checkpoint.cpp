#include "checkpoint.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>

namespace j1rt {

namespace {

bool read_file(const std::string& path, std::string& out, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = "reading " + path + ": cannot open";
    return false;
  }
  std::stringstream ss;
  ss << f.rdbuf();
  out = ss.str();
  return true;
}

bool read_json(const std::string& path, Json& out, std::string& err) {
  std::string text;
  if (!read_file(path, text, err)) return false;
  std::string perr;
  if (!parse_json(text, out, perr)) {
    err = "parsing " + path + ": " + perr;
    return false;
  }
  return true;
}

bool usize_of(const Json& v, const char* key, int& out, std::string& err) {
  const Json* x = v.get(key);
  if (!x || !x->is_num() || x->num < 0 || x->num != std::floor(x->num)) {
    err = std::string("config is missing ") + key;
    return false;
  }
  out = static_cast<int>(x->num);
  return true;
}

bool str_eq(const Json* v, const char* s) { return v && v->is_str() && v->str == s; }

}  // namespace

bool config_from_values(const Json& julia, const Json& enc, ModelConfig& cfg, std::string& err) {
  const Json* fv = julia.get("format_version");
  if (!fv || !fv->is_num() || fv->num != 1.0) {
    err = "Unsupported Julia checkpoint format";
    return false;
  }
  const Json* wd = julia.get("weight_dtype");
  if (wd && !(wd->is_str() && wd->str == "float32")) {
    err = "Only float32 Julia checkpoints are supported";
    return false;
  }
  if (!str_eq(enc.get("model_type"), "modernbert")) {
    err = "Encoder must be ModernBERT";
    return false;
  }
  for (const char* key : {"attention_bias", "mlp_bias", "norm_bias"}) {
    const Json* b = enc.get(key);
    if (!(b && b->is_bool() && !b->b)) {
      err = std::string("Unsupported encoder setting ") + key;
      return false;
    }
  }
  if (!str_eq(enc.get("hidden_activation"), "gelu")) {
    err = "Unsupported encoder activation";
    return false;
  }
  int hidden, heads, layers, every, local;
  if (!usize_of(enc, "hidden_size", hidden, err) || !usize_of(enc, "num_attention_heads", heads, err) ||
      !usize_of(enc, "num_hidden_layers", layers, err) || !usize_of(enc, "global_attn_every_n_layers", every, err) ||
      !usize_of(enc, "local_attention", local, err))
    return false;
  if (heads == 0 || hidden % heads != 0 || hidden / heads != 64) {
    err = "Runtime kernels require head_dim 64";
    return false;
  }
  if (every == 0) {
    err = "global_attn_every_n_layers must be positive";
    return false;
  }
  std::vector<std::string> types;
  const Json* lt = enc.get("layer_types");
  if (lt && lt->kind == Json::Array) {
    for (const auto& t : lt->arr) types.push_back(t.is_str() ? t.str : std::string());
  } else {
    for (int i = 0; i < layers; ++i) types.push_back(i % every == 0 ? "full_attention" : "sliding_attention");
  }
  if (static_cast<int>(types.size()) != layers) {
    err = "layer_types must list every layer";
    return false;
  }
  cfg.rope_theta.clear();
  for (const auto& kind : types) {
    const Json* rp = enc.get("rope_parameters");
    const Json* p = rp ? rp->get(kind) : nullptr;
    if (p) {
      if (!str_eq(p->get("rope_type"), "default")) {
        err = "Only default RoPE is supported";
        return false;
      }
      const Json* th = p->get("rope_theta");
      if (!th || !th->is_num()) {
        err = "rope_theta";
        return false;
      }
      cfg.rope_theta.push_back(static_cast<float>(th->num));
      continue;
    }
    const char* key = kind == "full_attention" ? "global_rope_theta" : "local_rope_theta";
    const Json* th = enc.get(key);
    if (!th || !th->is_num()) {
      err = std::string("missing ") + key;
      return false;
    }
    cfg.rope_theta.push_back(static_cast<float>(th->num));
  }
  int head_layers, inter, vocab, maxpos;
  if (!usize_of(julia, "head_layers", head_layers, err) || !usize_of(enc, "intermediate_size", inter, err) ||
      !usize_of(enc, "vocab_size", vocab, err) || !usize_of(enc, "max_position_embeddings", maxpos, err))
    return false;
  cfg.hidden = hidden;
  cfg.heads = heads;
  cfg.head_dim = hidden / heads;
  cfg.intermediate = inter;
  cfg.layers = layers;
  // ModernBertAttention: sliding iff layer_id % global_attn_every_n_layers != 0 (src/config.rs:84-85).
  cfg.global.assign(layers, false);
  for (int i = 0; i < layers; ++i) cfg.global[i] = (i % every == 0);
  cfg.half_window = local / 2;
  const Json* eps = enc.get("norm_eps");
  cfg.norm_eps = (eps && eps->is_num()) ? static_cast<float>(eps->num) : 1e-5f;
  cfg.vocab = vocab;
  cfg.max_positions = maxpos;
  cfg.head_layers = head_layers;
  cfg.head_heads = hidden / 64 > 1 ? hidden / 64 : 1;
  cfg.head_ff = 4 * hidden;
  return true;
}

bool config_load(const std::string& root, ModelConfig& cfg, std::string& err) {
  Json julia, enc;
  if (!read_json(root + "/julia_config.json", julia, err)) return false;
  if (!read_json(root + "/encoder/config.json", enc, err)) return false;
  return config_from_values(julia, enc, cfg, err);
}

void rope_table(float theta, int head_dim, int positions, std::vector<float>& cos_t, std::vector<float>& sin_t) {
  const int half = head_dim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i)
    inv[i] = 1.0f / std::pow(theta, static_cast<float>(2 * i) / static_cast<float>(head_dim));
  cos_t.assign(static_cast<size_t>(positions) * half, 0.f);
  sin_t.assign(static_cast<size_t>(positions) * half, 0.f);
  for (int p = 0; p < positions; ++p)
    for (int i = 0; i < half; ++i) {
      const float f = inv[i] * static_cast<float>(p);
      cos_t[static_cast<size_t>(p) * half + i] = std::cos(f);
      sin_t[static_cast<size_t>(p) * half + i] = std::sin(f);
    }
}

SafeTensors::~SafeTensors() {
  if (data_) munmap(const_cast<uint8_t*>(data_), size_);
}

bool SafeTensors::open(const std::string& path, std::string& err) {
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    err = "opening " + path + ": cannot open";
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    err = "opening " + path + ": stat failed";
    return false;
  }
  size_ = static_cast<size_t>(st.st_size);
  void* m = size_ ? mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
  ::close(fd);
  if (m == MAP_FAILED) {
    err = "mapping " + path + " failed";
    size_ = 0;
    return false;
  }
  data_ = static_cast<const uint8_t*>(m);
  static const char lfs[] = "version https://git-lfs.github.com/spec/v1";
  if (size_ >= sizeof(lfs) - 1 && std::memcmp(data_, lfs, sizeof(lfs) - 1) == 0) {
    err = "Checkpoint contains Git LFS pointers; fetch the real model weights first";
    return false;
  }
  if (size_ < 8) {
    err = "Truncated safetensors file";
    return false;
  }
  uint64_t n = 0;
  std::memcpy(&n, data_, 8);  // little-endian hosts only (x86-64 / aarch64)
  if (n > size_ - 8) {
    err = "Truncated safetensors header";
    return false;
  }
  Json header;
  std::string perr;
  if (!parse_json(std::string(reinterpret_cast<const char*>(data_ + 8), n), header, perr) ||
      header.kind != Json::Object) {
    err = "safetensors header: " + perr;
    return false;
  }
  for (const auto& kv : header.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& info = kv.second;
    if (!str_eq(info.get("dtype"), "F32")) {
      err = kv.first + ": only F32 tensors are supported";
      return false;
    }
    const Json* shape = info.get("shape");
    const Json* offs = info.get("data_offsets");
    if (!shape || shape->kind != Json::Array || !offs || offs->kind != Json::Array || offs->arr.size() != 2) {
      err = kv.first + ": bad header entry";
      return false;
    }
    Entry e;
    for (const auto& d : shape->arr) e.shape.push_back(static_cast<size_t>(d.num));
    const size_t a = static_cast<size_t>(offs->arr[0].num), b = static_cast<size_t>(offs->arr[1].num);
    if (!(a <= b && 8 + n + b <= size_)) {
      err = kv.first + ": data out of bounds";
      return false;
    }
    e.begin = 8 + n + a;
    e.end = 8 + n + b;
    tensors_[kv.first] = std::move(e);
  }
  return true;
}

const float* SafeTensors::f32(const std::string& name, const std::vector<size_t>& shape, std::string& err) {
  auto it = tensors_.find(name);
  if (it == tensors_.end()) {
    err = "missing tensor " + name;
    return nullptr;
  }
  const Entry& e = it->second;
  if (e.shape != shape) {
    std::string want, got;
    for (size_t d : shape) want += std::to_string(d) + ",";
    for (size_t d : e.shape) got += std::to_string(d) + ",";
    err = name + ": expected shape [" + want + "], found [" + got + "]";
    return nullptr;
  }
  size_t count = 1;
  for (size_t d : shape) count *= d;
  if (e.end - e.begin != count * 4) {
    err = name + ": byte size does not match shape";
    return nullptr;
  }
  const uint8_t* p = data_ + e.begin;
  if (reinterpret_cast<uintptr_t>(p) % 4 == 0) return reinterpret_cast<const float*>(p);
  scratch_.emplace_back(count);
  std::memcpy(scratch_.back().data(), p, count * 4);
  return scratch_.back().data();
}

}  // namespace j1rt
