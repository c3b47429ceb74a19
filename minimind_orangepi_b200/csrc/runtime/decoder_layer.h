// Decoder-layer weight and cache types with the reference's field names
// (src/csrc/models/minimind/decoder_layer.h:12-48). On the CUDA path the layer
// math runs inside libminimind_cuda.so; these host structs only carry fp32
// weights into the device upload and mirror per-layer cache lengths.
#pragma once

#include "config.h"

#include <cstdint>
#include <vector>

namespace minimind::model {

struct ExpertWeights {
  std::vector<float> gate_proj;
  std::vector<float> up_proj;
  std::vector<float> down_proj;
  std::vector<float> gate_up_proj;
};

struct DenseLayerWeights {
  std::vector<float> input_norm;
  std::vector<float> post_attention_norm;
  std::vector<float> q_norm;
  std::vector<float> k_norm;
  std::vector<float> q_proj;
  std::vector<float> k_proj;
  std::vector<float> v_proj;
  std::vector<float> qkv_proj;
  std::vector<float> o_proj;
  std::vector<float> gate_proj;
  std::vector<float> up_proj;
  std::vector<float> gate_up_proj;
  std::vector<float> down_proj;
  std::vector<float> moe_gate;
  std::vector<ExpertWeights> experts;
};

// Per-layer view of a sequence's cache. The K/V rows live in the device page
// pool; `tokens` mirrors the cached length like the reference's
// LayerKvCache::tokens. `keys`/`values` stay empty on the device path.
struct LayerKvCache {
  std::vector<float> keys;
  std::vector<float> values;
  int64_t tokens = 0;
};

}  // namespace minimind::model
