// Checkpoint access: the two JSON configs and the F32 safetensors file, with the
// reference's layout and checks (src/config.rs, src/weights.rs, src/model.rs).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "json.h"

namespace j1rt {

// ModelConfig (src/config.rs:6-24).
struct ModelConfig {
  int hidden = 0, heads = 0, head_dim = 0, intermediate = 0, layers = 0;
  std::vector<bool> global;       // per layer: full attention
  int half_window = 0;            // local_attention / 2
  std::vector<float> rope_theta;  // per layer RoPE base
  float norm_eps = 1e-5f;
  int vocab = 0, max_positions = 0;
  int head_layers = 0, head_heads = 0, head_ff = 0;
};

// ModelConfig::from_values (src/config.rs:43-96): same checks, same derived fields.
bool config_from_values(const Json& julia, const Json& enc, ModelConfig& cfg, std::string& err);
// ModelConfig::load (src/config.rs:36-40).
bool config_load(const std::string& root, ModelConfig& cfg, std::string& err);

// rope_table (src/config.rs:99-112): f32 inv_freq, f32 products, cos/sin; [positions, head_dim/2].
void rope_table(float theta, int head_dim, int positions, std::vector<float>& cos_t, std::vector<float>& sin_t);

// SafeTensors over a read-only memory map (src/weights.rs:51-89): F32 only, Git-LFS pointer check.
class SafeTensors {
 public:
  SafeTensors() = default;
  ~SafeTensors();
  SafeTensors(const SafeTensors&) = delete;
  SafeTensors& operator=(const SafeTensors&) = delete;

  bool open(const std::string& path, std::string& err);
  // Pointer to the tensor's F32 data after checking its shape; nullptr + err otherwise.
  // The data is 4-byte aligned in well-formed files; otherwise a copy is kept alive in `scratch_`.
  const float* f32(const std::string& name, const std::vector<size_t>& shape, std::string& err);
  bool has(const std::string& name) const { return tensors_.count(name) != 0; }

 private:
  struct Entry {
    std::vector<size_t> shape;
    size_t begin = 0, end = 0;
  };
  const uint8_t* data_ = nullptr;
  size_t size_ = 0;
  std::unordered_map<std::string, Entry> tensors_;
  std::vector<std::vector<float>> scratch_;
};

}  // namespace j1rt
